// bssm_internal.h -- declarations shared by the kernel translation units.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <string>

#include "bayes_ssm_b200.h"
#include "bssm_common.cuh"

namespace bssm {

// Fixed-dynamics constants (A = 0.97 I, Q = 0.1 I, R = 1), as in catid/bayes-ssm
// bayes_ssm/bayesian_layer.py:360-400.
constexpr float kFixedDecay = 0.97f;
constexpr float kFixedProcess = 0.1f;
constexpr float kFixedObservation = 1.0f;

template <typename TIn>
struct FwdArgs {
    const TIn *keys, *values, *queries;
    const float *decay, *process, *observation, *mean0, *cov0;
    float *out, *mean_final, *cov_final, *bmean, *bcov;
    float *rs;  // replay states (nullptr: not saved)
    long n, t;
    int chunks;
    float floor;
};

template <typename TIn>
struct BwdArgs {
    const TIn *keys, *values, *queries;
    const float *decay, *process, *observation, *mean0, *cov0;
    const float *bmean, *bcov, *gy, *gmf, *gcf;
    TIn *gk, *gv, *gq;
    float *ga, *gp, *gr, *gm0, *gc0;
    float *ws;
    const float *rs;  // replay states saved by the forward (nullptr: phase A recomputes them)
    long n, t;
    int chunks;
    float floor;
};

// Replay states: the state at every kReplaySpan-token boundary inside each
// chunk (not at the chunk start, which is the boundary checkpoint).  Layout
// per chain: [chunk][slot][mean D*M row-major | covariance upper triangle,
// row by row (tri_index) | pad].  The covariance is exactly symmetric in every
// kernel family, so its upper triangle is the whole state.
constexpr int kReplaySpan = 4;

// Position of covariance entry (i, j) in the row-by-row upper triangle.
__host__ __device__ constexpr int tri_index(int d, int i, int j) {
    return i <= j ? i * d - i * (i - 1) / 2 + (j - i) : j * d - j * (j - 1) / 2 + (i - j);
}
__host__ __device__ constexpr int tri_size(int d) { return d * (d + 1) / 2; }

// Row `row` of a covariance (D floats) to / from the packed upper triangle.
template <int D>
__device__ __forceinline__ void store_row_packed(float *packed, int row, const float (&v)[D]) {
#pragma unroll
    for (int j = 0; j < D; ++j)
        if (j >= row) packed[tri_index(D, row, j)] = v[j];
}
template <int D>
__device__ __forceinline__ void load_row_packed(const float *packed, int row, float (&v)[D]) {
#pragma unroll
    for (int j = 0; j < D; ++j) v[j] = packed[tri_index(D, row, j)];
}
__host__ __device__ inline long replay_slots_per_chunk(long t, int chunks) {
    const long span = chunks < t ? chunks : t;
    const long nsub = (span + kReplaySpan - 1) / kReplaySpan;
    return nsub > 1 ? nsub - 1 : 0;
}
// Floats per saved state, padded to a 16-byte multiple so that every slot
// starts 16-byte aligned (the lanes move it with 128-bit accesses).
__host__ __device__ constexpr int replay_state_floats(int d, int m) { return (d * m + tri_size(d) + 3) / 4 * 4; }
__host__ __device__ inline float *replay_slot(const float *rs, long chain, long nb, long slots, long ci,
                                              long j, int d, int m) {
    return const_cast<float *>(rs) + ((chain * nb + ci) * slots + (j - 1)) * static_cast<long>(replay_state_floats(d, m));
}

// Error reporting (thread-local message behind bssm_last_error()).
extern thread_local std::string g_last_error;
int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));

inline int check_launch(const char *what) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return fail(BSSM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
    g_last_error.clear();
    return BSSM_OK;
}

// Lane's CPL columns (col0 ..) of a row-major [D, M] mean in global memory.
template <int D, int M, int CPL>
__device__ __forceinline__ void load_mean_cols_g(const float *base, int col0, float (&Mc)[CPL][D]) {
#pragma unroll
    for (int i = 0; i < D; ++i) {
        float row[CPL];
        load_vec<CPL>(base + i * M + col0, row);
#pragma unroll
        for (int l = 0; l < CPL; ++l) Mc[l][i] = row[l];
    }
}
template <int D, int M, int CPL>
__device__ __forceinline__ void store_mean_cols_g(float *base, int col0, const float (&Mc)[CPL][D]) {
#pragma unroll
    for (int i = 0; i < D; ++i) {
        float row[CPL];
#pragma unroll
        for (int l = 0; l < CPL; ++l) row[l] = Mc[l][i];
        store_vec<CPL>(base + i * M + col0, row);
    }
}

// Coherent vector load, for data the same kernel wrote earlier (the phase-A
// workspace): ld.global, never the read-only path.
template <int N>
__device__ __forceinline__ void load_vec_coherent(const float *p, float (&o)[N]) {
    static_assert(N % 4 == 0, "width");
#pragma unroll
    for (int i = 0; i < N; i += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(p + i);
        o[i] = v.x; o[i + 1] = v.y; o[i + 2] = v.z; o[i + 3] = v.w;
    }
}

// Shared-memory-staged kernels (bssm_staged.cu).
template <typename TIn> bool staged_supported(int d);
template <typename TIn> int staged_forward(int d, int fixed, const FwdArgs<TIn> &a, cudaStream_t st);
template <typename TIn>
int staged_backward(int d, int fixed, bool dyn, bool init, const BwdArgs<TIn> &a, cudaStream_t st);

// Thread-per-chain kernels (bssm_chain.cu): shapes with 16-byte rows and
// T, chunk length multiples of kReplaySpan.  The backward needs the forward's
// replay states whenever a chunk is longer than kReplaySpan tokens.
template <typename TIn> bool chain_eligible(int d, long n, long t, int chunks);
template <typename TIn> int chain_forward(int d, int fixed, const FwdArgs<TIn> &a, cudaStream_t st);
template <typename TIn>
int chain_backward(int d, int fixed, bool dyn, bool init, const BwdArgs<TIn> &a, cudaStream_t st);

}  // namespace bssm
