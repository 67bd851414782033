// bssm_internal.h -- declarations shared by the kernel translation units.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <string>
#include <type_traits>

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

// Replay buffer, part one -- replay states: the state at every
// kReplaySpan-token boundary inside each chunk (not at the chunk start, which
// is the boundary checkpoint).  A state is [mean D*M row-major | covariance
// upper triangle, row by row (tri_index) | pad] (the covariance is exactly
// symmetric in every kernel family, so its upper triangle is the whole
// state).  States are stored as a structure of arrays of float quads over
// groups of 32 chains: float f of state (chunk ci, slot j) of chain c is at
//     (((((c / 32) * nb + ci) * slots + j - 1) * SF / 4 + f / 4) * 32 + c % 32) * 4 + f % 4,
// so quad f / 4 of a group's 32 chains is one contiguous 512-byte line: a
// warp moves it with one 16-byte access per lane.
constexpr int kReplaySpan = 4;

// Position of covariance entry (i, j) in the row-by-row upper triangle.
__host__ __device__ constexpr int tri_index(int d, int i, int j) {
    return i <= j ? i * d - i * (i - 1) / 2 + (j - i) : j * d - j * (j - 1) / 2 + (i - j);
}
__host__ __device__ constexpr int tri_size(int d) { return d * (d + 1) / 2; }

__host__ __device__ inline long replay_slots_per_chunk(long t, int chunks) {
    const long span = chunks < t ? chunks : t;
    const long nsub = (span + kReplaySpan - 1) / kReplaySpan;
    return nsub > 1 ? nsub - 1 : 0;
}
// Floats per state, a multiple of 4.
__host__ __device__ constexpr int replay_state_floats(int d, int m) { return (d * m + tri_size(d) + 3) / 4 * 4; }
__host__ __device__ inline long replay_groups(long n) { return (n + 31) / 32; }
// Index of float 0 of chain `chain`'s state (ci, j >= 1); float f is at
// rs_at(base, f).
__host__ __device__ inline long replay_state_base(long chain, long nb, long slots, long ci, long j, int sf) {
    return (((((chain >> 5) * nb + ci) * slots + (j - 1)) * (sf / 4)) * 32 + (chain & 31)) * 4;
}
__host__ __device__ constexpr long rs_at(long base, int f) { return base + (f >> 2) * 128 + (f & 3); }
// Floats of the state part of the buffer.
__host__ __device__ inline long replay_state_part(long n, long t, int chunks, int d, int m) {
    const long nb = (t + chunks - 1) / chunks;
    return replay_groups(n) * 32 * nb * replay_slots_per_chunk(t, chunks) * replay_state_floats(d, m);
}

// A lane's mean columns / a covariance row to or from a state (base from
// replay_state_base).
template <int D, int M, int CPL>
__device__ __forceinline__ void rs_put_mean_cols(float *rs, long base, int col0, const float (&Mc)[CPL][D]) {
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int l = 0; l < CPL; ++l) rs[rs_at(base, i * M + col0 + l)] = Mc[l][i];
}
template <int D, int M, int CPL>
__device__ __forceinline__ void rs_get_mean_cols(const float *rs, long base, int col0, float (&Mc)[CPL][D]) {
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int l = 0; l < CPL; ++l) Mc[l][i] = rs[rs_at(base, i * M + col0 + l)];
}
template <int D, int M>
__device__ __forceinline__ void rs_put_row(float *rs, long base, int row, const float (&v)[D]) {
#pragma unroll
    for (int j = 0; j < D; ++j)
        if (j >= row) rs[rs_at(base, D * M + tri_index(D, row, j))] = v[j];
}
template <int D, int M>
__device__ __forceinline__ void rs_get_row(const float *rs, long base, int row, float (&v)[D]) {
#pragma unroll
    for (int j = 0; j < D; ++j) v[j] = rs[rs_at(base, D * M + tri_index(D, row, j))];
}

// After the states, the replay buffer holds every token's gain u [N][T][D]
// as the forward computed it, then its signed gain scale [N][T]: beta when
// s >= floor (the clamp passes the gradient to s), -beta when not.  beta is
// positive or NaN, so the sign carries the clamp mask and |.| the value; a
// NaN s gives -NaN, masked as s >= floor would.  Each part starts 16-byte
// aligned.  With them a backward replays the mean without waiting for the
// covariance replay.
__host__ __device__ inline long round4(long x) { return (x + 3) / 4 * 4; }
__host__ __device__ inline float *replay_gains(const float *rs, long n, long t, int chunks, int d, int m) {
    return const_cast<float *>(rs) + replay_state_part(n, t, chunks, d, m);
}
__host__ __device__ inline float *replay_gain_scales(const float *rs, long n, long t, int chunks, int d, int m) {
    return replay_gains(rs, n, t, chunks, d, m) + round4(n * t * d);
}
// Floats of the whole replay buffer.
__host__ __device__ inline long replay_floats(long n, long t, int chunks, int d, int m) {
    return replay_state_part(n, t, chunks, d, m) + round4(n * t * d) + round4(n * t);
}
__device__ __forceinline__ float signed_gain_scale(float beta, float s, float floor_) {
    return s >= floor_ ? beta : -beta;
}
__device__ __forceinline__ bool gain_scale_passes(float bt) { return !signbit(bt); }

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
template <typename TIn> bool chain_eligible(int d, long n, long t, int chunks, bool forward);
// Key dim 64 x value dim 64, float32 (bssm_d64.cu): one CTA per chain.
int d64_forward(int fixed, const FwdArgs<float> &a, cudaStream_t st);
int d64_backward(int fixed, bool dyn, bool init, const BwdArgs<float> &a, cudaStream_t st);
size_t d64_workspace_bytes(long n, long t, int chunks);
template <typename TIn> int chain_forward(int d, int fixed, const FwdArgs<TIn> &a, cudaStream_t st);
template <typename TIn>
int chain_backward(int d, int fixed, bool dyn, bool init, const BwdArgs<TIn> &a, cudaStream_t st);

}  // namespace bssm
