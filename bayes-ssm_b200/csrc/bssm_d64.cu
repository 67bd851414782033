// bssm_d64.cu -- the chunked forward and replay backward at key dim 64 x
// value dim 64 (catid/bayes-ssm bayes_ssm/persistent_bayes_chunked.cu:176-434,
// the D64M64 variant loaded by bayes_ssm/fused_cuda.py:33-44).
//
// Same recurrence and adjoint as the D <= 8 families (bayesian_layer.py:153-181;
// the covariance adjoint is kept exactly symmetric, which is also the
// reference's D64 convention, persistent_bayes_chunked.cu:332).  The state is
// 64 x 64 mean plus 64 x 64 covariance per chain, so one CTA of 256 threads
// serves one chain and every thread owns a 4 x 4 tile of each matrix:
//
// * thread t = 16 r + c (r, c in 0..15): covariance tile P[4r + i][4c + j] and
//   mean tile M[4c + i][4r + j] (rows = key index, columns = value index).
//   The mean tile is placed transposed on purpose: the 16 threads of one
//   half-warp share r, so every contraction over the key index -- the gain
//   u = P'k (over the covariance's columns), the innovation e = v - (AM)^T k
//   and the readout y = M^T q (over the mean's rows) -- is a 4-value
//   butterfly inside the half-warp, with no shared memory.
// * Per token, only the gain u (64 floats) and the 16 partial sums of k.u
//   cross half-warps, through shared memory: two barriers per token.
// * Token inputs are staged by cp.async, two tokens ahead.
//
// Backward (recompute mode, one launch): per chunk, last to first, the chunk
// is replayed from its boundary checkpoint and the state at the start of
// every kSub-token sub-chunk is saved to the caller's workspace; then per
// sub-chunk, last to first, the sub-chunk is replayed once more with every
// token's pre-step tiles kept in shared memory (thread-private slots) and the
// reverse step runs over it.  Contractions over the value index (the readout
// gradient, h = gM e, M ge and the mean part of the decay gradient) cross
// half-warps and go through one shared-memory reduction per token.
//
// FP32 inputs only (the reference's D64 path is FP32).  The kernels keep the
// covariance exactly symmetric: every product that fills entry (i, j) is formed
// from commutative pairs, so the two tiles holding (i, j) and (j, i) agree bit
// for bit.
#include <cuda_runtime.h>

#include <cstdint>

#include "bayes_ssm_b200.h"
#include "bssm_common.cuh"
#include "bssm_internal.h"

namespace bssm {
namespace d64 {

constexpr int D = 64, M = 64;
constexpr int kThreads = 256;
constexpr int kSub = 2;           // backward sub-chunk: tokens of history in shared memory
constexpr int kStages = 3;        // forward input ring (two tokens ahead)
constexpr int kTileFloats = 16;   // per thread and matrix
constexpr int kStateFloats = 2 * kTileFloats * kThreads;  // one saved state (P and M tiles)

// One token's inputs in shared memory.
struct TokIn {
    float k[D], q[D], a[D], v[D], gy[M];
    float p, r, pad[2];
};

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void st4(float *p, float x, float y, float z, float w) {
    *reinterpret_cast<float4 *>(p) = make_float4(x, y, z, w);
}
__device__ __forceinline__ void unpack(const float4 v, float (&o)[4]) {
    o[0] = v.x;
    o[1] = v.y;
    o[2] = v.z;
    o[3] = v.w;
}

// Half-warp sums over the 16 lanes c = 0..15 (lane bits 3..0).  A butterfly
// on every value would take 4 shuffles per value; these first scatter the
// values over the lanes (at each of the two top levels a lane keeps half of
// its values and sends the other half), so each sum is formed once, and the
// lanes that need every sum gather them back.  Every lane holding a sum holds
// the same bits, which keeps the covariance tiles exactly symmetric.
__device__ __forceinline__ float shx(float v, int o) { return __shfl_xor_sync(0xffffffffu, v, o); }
template <int N>
__device__ __forceinline__ float pick(const float (&a)[N], int i) {
    static_assert(N == 4, "four values");
    return (i & 2) ? ((i & 1) ? a[3] : a[2]) : ((i & 1) ? a[1] : a[0]);
}

// Sum of value (c >> 2) & 3 of 4 values, in every lane of that group of four
// lanes (5 shuffles instead of 16).
__device__ __forceinline__ float hw_scatter4(const float (&x)[4]) {
    const bool b3 = threadIdx.x & 8, b2 = threadIdx.x & 4;
    float y[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) y[i] = (b3 ? x[2 + i] : x[i]) + shx(b3 ? x[i] : x[2 + i], 8);
    float z = (b2 ? y[1] : y[0]) + shx(b2 ? y[0] : y[1], 4);
    z += shx(z, 2);
    z += shx(z, 1);
    return z;
}

// Sums of 4 values, all of them in every lane (8 shuffles instead of 16).
__device__ __forceinline__ void hw_sum4(float (&x)[4]) {
    const bool b3 = threadIdx.x & 8, b2 = threadIdx.x & 4;
    const float z = hw_scatter4(x), o = shx(z, 4);
    const float y0 = b2 ? o : z, y1 = b2 ? z : o;  // values 2 b3 and 2 b3 + 1
    const float p0 = shx(y0, 8), p1 = shx(y1, 8);
    x[0] = b3 ? p0 : y0;
    x[1] = b3 ? p1 : y1;
    x[2] = b3 ? y0 : p0;
    x[3] = b3 ? y1 : p1;
}

// Sums of 8 values, all of them in every lane (15 shuffles instead of 32).
__device__ __forceinline__ void hw_sum8(float (&x)[8]) {
    const bool b3 = threadIdx.x & 8, b2 = threadIdx.x & 4, b1 = threadIdx.x & 2;
    float y[4], z[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) y[i] = (b3 ? x[4 + i] : x[i]) + shx(b3 ? x[i] : x[4 + i], 8);
#pragma unroll
    for (int i = 0; i < 2; ++i) z[i] = (b2 ? y[2 + i] : y[i]) + shx(b2 ? y[i] : y[2 + i], 4);
    float w = (b1 ? z[1] : z[0]) + shx(b1 ? z[0] : z[1], 2);
    w += shx(w, 1);  // value 4 b3 + 2 b2 + b1
    const float w2 = shx(w, 2);
    z[0] = b1 ? w2 : w;
    z[1] = b1 ? w : w2;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float o = shx(z[i], 4);
        y[i] = b2 ? o : z[i];
        y[2 + i] = b2 ? z[i] : o;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float o = shx(y[i], 8);
        x[i] = b3 ? o : y[i];
        x[4 + i] = b3 ? y[i] : o;
    }
}

__device__ __forceinline__ float clamp_beta(float s, float floor_) { return 1.0f / (s < floor_ ? floor_ : s); }

// Stage token `ti`'s inputs of chain `chain` (threads 0..79 issue the copies).
template <bool FIXED, bool WANT_Q, bool WANT_GY>
__device__ __forceinline__ void stage_token(TokIn *dst, const BwdArgs<float> &A, long chain, long ti) {
    const int t = threadIdx.x;
    const long row = chain * A.t + ti;
    const uint32_t base = smem_u32(dst);
    if (t < 16) {
        cp_async<16>(base + offsetof(TokIn, k) + 16 * t, A.keys + row * D + 4 * t);
    } else if (t < 32) {
        if (WANT_Q) cp_async<16>(base + offsetof(TokIn, q) + 16 * (t - 16), A.queries + row * D + 4 * (t - 16));
    } else if (t < 48) {
        if (!FIXED) cp_async<16>(base + offsetof(TokIn, a) + 16 * (t - 32), A.decay + row * D + 4 * (t - 32));
    } else if (t < 64) {
        cp_async<16>(base + offsetof(TokIn, v) + 16 * (t - 48), A.values + row * M + 4 * (t - 48));
    } else if (t < 80) {
        if (WANT_GY && A.gy != nullptr) cp_async<16>(base + offsetof(TokIn, gy) + 16 * (t - 64), A.gy + row * M + 4 * (t - 64));
    } else if (t == 80) {
        if (!FIXED) cp_async<4>(base + offsetof(TokIn, p), A.process + row);
    } else if (t == 81) {
        if (!FIXED) cp_async<4>(base + offsetof(TokIn, r), A.observation + row);
    }
}

// Constants that FIXED dynamics replace, and zero gy when none is given.
template <bool FIXED, bool WANT_GY>
__device__ __forceinline__ void fill_constants(TokIn *dst, const BwdArgs<float> &A) {
    const int t = threadIdx.x;
    if (FIXED) {
        if (t < D) dst->a[t] = kFixedDecay;
        if (t == 0) {
            dst->p = kFixedProcess;
            dst->r = kFixedObservation;
        }
    }
    if (WANT_GY && A.gy == nullptr && t < M) dst->gy[t] = 0.f;
}

// Per-thread state: covariance tile and (transposed) mean tile.
struct Tiles {
    float P[4][4];  // P[4r + i][4c + j]
    float Mt[4][4];  // M[4c + i][4r + j]
};

__device__ __forceinline__ void load_state_g(Tiles &s, const float *mean, const float *cov, int r, int c) {
    // mean NULL: zeros; cov NULL: identity; the covariance enters symmetrised
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float m4[4], a4[4], b4[4];
        if (mean) {
            unpack(ld4(mean + (4 * c + i) * M + 4 * r), m4);
        } else {
            m4[0] = m4[1] = m4[2] = m4[3] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) s.Mt[i][j] = m4[j];
        if (cov) {
            unpack(ld4(cov + (4 * r + i) * D + 4 * c), a4);
#pragma unroll
            for (int j = 0; j < 4; ++j) b4[j] = cov[(4 * c + j) * D + 4 * r + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) s.P[i][j] = 0.5f * (a4[j] + b4[j]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) s.P[i][j] = (r == c && i == j) ? 1.f : 0.f;
        }
    }
}
__device__ __forceinline__ void store_state_g(const Tiles &s, float *mean, float *cov, int r, int c) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        st4(cov + (4 * r + i) * D + 4 * c, s.P[i][0], s.P[i][1], s.P[i][2], s.P[i][3]);
        st4(mean + (4 * c + i) * M + 4 * r, s.Mt[i][0], s.Mt[i][1], s.Mt[i][2], s.Mt[i][3]);
    }
}
// Thread-tile layout of a saved state: quad x (rows of P, then of Mt) of
// thread t at (x * 256 + t) * 4, so a warp moves 512 contiguous bytes per
// 16-byte access.
__device__ __forceinline__ void store_state_ws(const Tiles &s, float *ws) {
    float4 *const w = reinterpret_cast<float4 *>(ws) + threadIdx.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        w[i * kThreads] = make_float4(s.P[i][0], s.P[i][1], s.P[i][2], s.P[i][3]);
        w[(4 + i) * kThreads] = make_float4(s.Mt[i][0], s.Mt[i][1], s.Mt[i][2], s.Mt[i][3]);
    }
}
__device__ __forceinline__ void load_state_ws(Tiles &s, const float *ws) {
    const float4 *const w = reinterpret_cast<const float4 *>(ws) + threadIdx.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        unpack(w[i * kThreads], s.P[i]);
        unpack(w[(4 + i) * kThreads], s.Mt[i]);
    }
}

// Exchange buffers of one token (double-buffered by token parity).
struct __align__(16) Xchg {
    float u[2][D];
    float spart[2][16];
};

// Gain, innovation and scale of one token; the exchange happens inside (one
// barrier).  Returns beta; u_r / u_c are the gain at rows 4r.. / 4c..,
// e_r the innovation at value columns 4r...
struct StepOut {
    float u_r[4], u_c[4], e_r[4];
    float beta, s;
};

__device__ __forceinline__ void gain_pre(const Tiles &st, const TokIn &tk, Xchg &x, int par, int r, int c,
                                         StepOut &o) {
    float k_c[4], a_c[4], k_r[4], a_r[4], v_r[4];
    unpack(ld4(tk.k + 4 * c), k_c);
    unpack(ld4(tk.a + 4 * c), a_c);
    unpack(ld4(tk.k + 4 * r), k_r);
    unpack(ld4(tk.a + 4 * r), a_r);
    unpack(ld4(tk.v + 4 * r), v_r);
    float w_c[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) w_c[j] = a_c[j] * k_c[j];
    float pu[4], pe[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float z = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) z = fmaf(st.P[i][j], w_c[j], z);
        pu[i] = z;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float z = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) z = fmaf(st.Mt[i][j], w_c[i], z);
        pe[j] = z;
    }
    float pue[8] = {pu[0], pu[1], pu[2], pu[3], pe[0], pe[1], pe[2], pe[3]};
    hw_sum8(pue);
    const float p = tk.p;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        o.u_r[i] = fmaf(a_r[i], pue[i], p * k_r[i]);
        o.e_r[i] = v_r[i] - pue[4 + i];
    }
    if (c == 0) {
        st4(x.u[par] + 4 * r, o.u_r[0], o.u_r[1], o.u_r[2], o.u_r[3]);
        float sp = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) sp = fmaf(k_r[i], o.u_r[i], sp);
        x.spart[par][r] = sp;
    }
}
// The rest once the exchange is visible (after a block barrier).
__device__ __forceinline__ void gain_post(const TokIn &tk, const Xchg &x, int par, int c, float floor_, StepOut &o) {
    float s = tk.r;
#pragma unroll
    for (int q = 0; q < 16; q += 4) {  // in order, four at a time
        const float4 v = ld4(x.spart[par] + q);
        s = ((s + v.x) + v.y + v.z) + v.w;
    }
    o.s = s;
    o.beta = clamp_beta(s, floor_);
    unpack(ld4(x.u[par] + 4 * c), o.u_c);
}

__device__ __forceinline__ void gain_step(const Tiles &st, const TokIn &tk, Xchg &x, int par, int r, int c,
                                          float floor_, StepOut &o) {
    gain_pre(st, tk, x, par, r, c, o);
    __syncthreads();
    gain_post(tk, x, par, c, floor_, o);
}

// The state update of one token from its gain (in place).
__device__ __forceinline__ void update_step(Tiles &st, const TokIn &tk, const StepOut &o, int r, int c) {
    float a_c[4], a_r[4];
    unpack(ld4(tk.a + 4 * c), a_c);
    unpack(ld4(tk.a + 4 * r), a_r);
    const float p = tk.p, beta = o.beta;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            // P' = a_i a_j P + p delta - beta (u_i u_j): each factor pair commutes
            float v = (a_r[i] * a_c[j]) * st.P[i][j];
            if (r == c && i == j) v += p;
            st.P[i][j] = fmaf(-beta, o.u_r[i] * o.u_c[j], v);
        }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float bu = beta * o.u_c[i];
#pragma unroll
        for (int j = 0; j < 4; ++j) st.Mt[i][j] = fmaf(bu, o.e_r[j], a_c[i] * st.Mt[i][j]);
    }
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <bool FIXED>
__global__ void __launch_bounds__(kThreads, 2) d64_forward(const FwdArgs<float> F) {
    __shared__ __align__(16) TokIn ring[kStages];
    __shared__ __align__(16) Xchg x;
    const long chain = blockIdx.x;
    const int t = threadIdx.x, r = t >> 4, c = t & 15;
    const long T = F.t;
    const int L = F.chunks;
    const long nb = (T + L - 1) / L;
    // the staging helper reads through the backward's argument record
    BwdArgs<float> A{};
    A.keys = F.keys;
    A.values = F.values;
    A.queries = F.queries;
    A.decay = F.decay;
    A.process = F.process;
    A.observation = F.observation;
    A.t = F.t;
    Tiles st;
    load_state_g(st, F.mean0 ? F.mean0 + chain * D * M : nullptr, F.cov0 ? F.cov0 + chain * D * D : nullptr, r, c);
    store_state_g(st, F.bmean + chain * (nb + 1) * D * M, F.bcov + chain * (nb + 1) * D * D, r, c);
#pragma unroll
    for (int s = 0; s < kStages; ++s) fill_constants<FIXED, false>(ring + s, A);
    // One block barrier per token: the gain exchange's barrier of token ti also
    // publishes token ti + 1 (each thread waits for its own copies of it first)
    // and frees the slot of token ti - 1 for token ti + 2.
    for (long ti = 0; ti < 2 && ti < T; ++ti) {
        stage_token<FIXED, true, false>(ring + ti, A, chain, ti);
        cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();  // tokens 0 and 1 visible
    for (long ti = 0; ti < T; ++ti) {
        const int slot = static_cast<int>(ti % kStages);
        const TokIn &tk = ring[slot];
        StepOut o;
        gain_pre(st, tk, x, static_cast<int>(ti & 1), r, c, o);
        cp_async_wait<0>();  // this thread's copies of token ti + 1
        __syncthreads();     // exchange and token ti + 1 visible; every thread is done with token ti - 1
        if (ti + 2 < T) {
            stage_token<FIXED, true, false>(ring + (ti + 2) % kStages, A, chain, ti + 2);
            cp_async_commit();
        }
        gain_post(tk, x, static_cast<int>(ti & 1), c, F.floor, o);
        update_step(st, tk, o, r, c);
        // readout y = M'^T q over the key rows 4c.. of the tile, then the half-warp
        float q_c[4], py[4];
        unpack(ld4(tk.q + 4 * c), q_c);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float z = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) z = fmaf(st.Mt[i][j], q_c[i], z);
            py[j] = z;
        }
        const float yv = hw_scatter4(py);  // y at value column 4r + ((c >> 2) & 3)
        if ((c & 3) == 0) F.out[(chain * T + ti) * M + 4 * r + ((c >> 2) & 3)] = yv;
        if ((ti + 1) % L == 0 || ti + 1 == T) {
            const long b = (ti + 1 + L - 1) / L;
            store_state_g(st, F.bmean + (chain * (nb + 1) + b) * D * M, F.bcov + (chain * (nb + 1) + b) * D * D, r,
                          c);
        }
    }
    store_state_g(st, F.mean_final + chain * D * M, F.cov_final + chain * D * D, r, c);
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
// Shared memory of the backward (dynamic).
struct BwdSmem {
    TokIn tok[kSub];                     // the sub-chunk's inputs
    TokIn ring[kStages];                 // phase-A input ring
    Xchg x;
    float4 hist[kSub][2 * kTileFloats / 4][kThreads];  // pre-step tile rows, thread-private columns
    float hu[kSub][D], he[kSub][M];      // per-token gain and innovation
    float hbeta[kSub], hs[kSub];
    float red[4][16][D];                 // value-index partial sums: gq, h, M ge, gMbar . M
    float fin[4][D];                     // their totals
    float ru[2][D];                      // R u (by token parity)
    float urup[2][16];                   // partial u . R u
    float trp[kSub][16];                 // partial traces of the symmetric covariance adjoint
};

// Two CTAs per SM (registers capped at 128, a few bytes spilled in three of
// the eight instantiations): the backward is bound by its barriers, so a second
// chain per SM helps (B256 T512 H8: 24.9 -> 19.8 ms against one CTA at 189
// registers).
#ifndef BSSM_D64_BWD_MINB
#define BSSM_D64_BWD_MINB 2
#endif
template <bool FIXED, bool NEED_DYN, bool NEED_INIT>
__global__ void __launch_bounds__(kThreads, BSSM_D64_BWD_MINB) d64_backward(const BwdArgs<float> A) {
    extern __shared__ __align__(16) char smem_raw[];
    BwdSmem &sm = *reinterpret_cast<BwdSmem *>(smem_raw);
    const long chain = blockIdx.x;
    const int t = threadIdx.x, r = t >> 4, c = t & 15;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;
    const int nsub_max = (static_cast<int>(L < T ? L : T) + kSub - 1) / kSub;
    float *const ws = A.ws + chain * static_cast<long>(nsub_max > 1 ? nsub_max - 1 : 0) * kStateFloats;
    const float floor_ = A.floor;

    // adjoint state: gM (mean layout), R (covariance layout, symmetric)
    float gM[4][4], R[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float m4[4] = {0.f, 0.f, 0.f, 0.f};
        if (A.gmf) unpack(ld4(A.gmf + chain * D * M + (4 * c + i) * M + 4 * r), m4);
#pragma unroll
        for (int j = 0; j < 4; ++j) gM[i][j] = m4[j];
        if (A.gcf) {
            const float *g = A.gcf + chain * D * D;
#pragma unroll
            for (int j = 0; j < 4; ++j) R[i][j] = 0.5f * (g[(4 * r + i) * D + 4 * c + j] + g[(4 * c + j) * D + 4 * r + i]);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) R[i][j] = 0.f;
        }
    }
#pragma unroll
    for (int s = 0; s < kStages; ++s) fill_constants<FIXED, false>(sm.ring + s, A);
#pragma unroll
    for (int s = 0; s < kSub; ++s) fill_constants<FIXED, true>(sm.tok + s, A);
    __syncthreads();

    for (long ci = nb - 1; ci >= 0; --ci) {
        const long t0 = ci * L;
        const int len = static_cast<int>(L < T - t0 ? L : T - t0);
        const int nsub = (len + kSub - 1) / kSub;
        const float *bmean = A.bmean + (chain * (nb + 1) + ci) * D * M;
        const float *bcov = A.bcov + (chain * (nb + 1) + ci) * D * D;
        Tiles st;
        // ---- phase A: replay the chunk, saving the state at each sub-chunk start
        if (nsub > 1) {
            load_state_g(st, bmean, bcov, r, c);
            const int upto = (nsub - 1) * kSub;  // tokens to replay
            // one block barrier per token, as in the forward
            for (int li = 0; li < 2 && li < upto; ++li) {
                stage_token<FIXED, false, false>(sm.ring + li, A, chain, t0 + li);
                cp_async_commit();
            }
            cp_async_wait<0>();
            __syncthreads();
            for (int li = 0; li < upto; ++li) {
                const TokIn &tk = sm.ring[li % kStages];
                StepOut o;
                gain_pre(st, tk, sm.x, li & 1, r, c, o);
                cp_async_wait<0>();  // this thread's copies of token li + 1
                __syncthreads();     // exchange and token li + 1 visible; token li - 1 done with
                if (li + 2 < upto) {
                    stage_token<FIXED, false, false>(sm.ring + (li + 2) % kStages, A, chain, t0 + li + 2);
                    cp_async_commit();
                }
                gain_post(tk, sm.x, li & 1, c, floor_, o);
                update_step(st, tk, o, r, c);
                if ((li + 1) % kSub == 0) store_state_ws(st, ws + static_cast<long>((li + 1) / kSub - 1) * kStateFloats);
            }
        }
        // ---- per sub-chunk, last to first: replay with history, then the reverse step
        for (int sb = nsub - 1; sb >= 0; --sb) {
            const int s0 = sb * kSub;
            const int slen = len - s0 < kSub ? len - s0 : kSub;
            __syncthreads();  // the previous sub-chunk is done with tok[] and the history
            for (int x = 0; x < slen; ++x) stage_token<FIXED, true, true>(sm.tok + x, A, chain, t0 + s0 + x);
            cp_async_commit();
            if (sb == 0) {
                load_state_g(st, bmean, bcov, r, c);
            } else {
                __threadfence_block();
                load_state_ws(st, ws + static_cast<long>(sb - 1) * kStateFloats);
            }
            cp_async_wait<0>();
            __syncthreads();
            for (int x = 0; x < slen; ++x) {
                const TokIn &tk = sm.tok[x];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    sm.hist[x][i][t] = make_float4(st.P[i][0], st.P[i][1], st.P[i][2], st.P[i][3]);
                    sm.hist[x][4 + i][t] = make_float4(st.Mt[i][0], st.Mt[i][1], st.Mt[i][2], st.Mt[i][3]);
                }
                StepOut o;
                gain_step(st, tk, sm.x, x & 1, r, c, floor_, o);
                if (c == 0) {
                    st4(sm.hu[x] + 4 * r, o.u_r[0], o.u_r[1], o.u_r[2], o.u_r[3]);
                    st4(sm.he[x] + 4 * r, o.e_r[0], o.e_r[1], o.e_r[2], o.e_r[3]);
                }
                if (t == 0) {
                    sm.hbeta[x] = o.beta;
                    sm.hs[x] = o.s;
                }
                update_step(st, tk, o, r, c);
            }
            __syncthreads();  // history complete
            // ---- reverse step over the sub-chunk
            for (int x = slen - 1; x >= 0; --x) {
                const TokIn &tk = sm.tok[x];
                const long row = chain * T + t0 + s0 + x;
                const int par = x & 1;
                float Pp[4][4], Mp[4][4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    unpack(sm.hist[x][i][t], Pp[i]);
                    unpack(sm.hist[x][4 + i][t], Mp[i]);
                }
                float k_c[4], a_c[4], q_c[4], k_r[4], a_r[4], gy_r[4], u_c[4], u_r[4], e_r[4];
                unpack(ld4(tk.k + 4 * c), k_c);
                unpack(ld4(tk.a + 4 * c), a_c);
                unpack(ld4(tk.q + 4 * c), q_c);
                unpack(ld4(tk.k + 4 * r), k_r);
                unpack(ld4(tk.a + 4 * r), a_r);
                unpack(ld4(tk.gy + 4 * r), gy_r);
                unpack(ld4(sm.hu[x] + 4 * c), u_c);
                unpack(ld4(sm.hu[x] + 4 * r), u_r);
                unpack(ld4(sm.he[x] + 4 * r), e_r);
                const float beta = sm.hbeta[x], s = sm.hs[x], p = tk.p;
                // mean side (rows 4c.., value columns 4r..)
                float gMn[4][4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) gMn[i][j] = fmaf(q_c[i], gy_r[j], gM[i][j]);
                float ge[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float z = 0.f;
#pragma unroll
                    for (int i = 0; i < 4; ++i) z = fmaf(gMn[i][j], u_c[i], z);
                    ge[j] = z;
                }
                hw_sum4(ge);
#pragma unroll
                for (int j = 0; j < 4; ++j) ge[j] *= beta;
                float pq[4], ph[4], pm[4], pg[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float zq = 0.f, zh = 0.f, zm = 0.f, zg = 0.f;
                    const float bu = beta * u_c[i];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        // post-step mean, as the forward formed it
                        const float mn = fmaf(bu, e_r[j], a_c[i] * Mp[i][j]);
                        zq = fmaf(mn, gy_r[j], zq);
                        zh = fmaf(gMn[i][j], e_r[j], zh);
                        zm = fmaf(Mp[i][j], ge[j], zm);
                        const float gmb = fmaf(-k_c[i], ge[j], gMn[i][j]);
                        zg = fmaf(gmb, Mp[i][j], zg);
                        gM[i][j] = a_c[i] * gmb;  // gradient of the pre-step mean
                    }
                    pq[i] = zq;
                    ph[i] = zh;
                    pm[i] = zm;
                    pg[i] = zg;
                }
                st4(&sm.red[0][r][4 * c], pq[0], pq[1], pq[2], pq[3]);
                st4(&sm.red[1][r][4 * c], ph[0], ph[1], ph[2], ph[3]);
                st4(&sm.red[2][r][4 * c], pm[0], pm[1], pm[2], pm[3]);
                st4(&sm.red[3][r][4 * c], pg[0], pg[1], pg[2], pg[3]);
                // covariance side: R u over the columns 4c..
                float ru[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float z = 0.f;
#pragma unroll
                    for (int j = 0; j < 4; ++j) z = fmaf(R[i][j], u_c[j], z);
                    ru[i] = z;
                }
                {
                    // (R u) at row 4r + ((c >> 2) & 3) and the half-warp's u . R u
                    const int ri = (c >> 2) & 3;
                    const float rv = hw_scatter4(ru);
                    if ((c & 3) == 0) sm.ru[par][4 * r + ri] = rv;
                    float uru = pick(u_r, ri) * rv;
                    uru += shx(uru, 4);
                    uru += shx(uru, 8);
                    if (c == 0) sm.urup[par][r] = uru;
                }
                if (c == 0) {  // gv = ge at value columns 4r..
                    st4(A.gv + row * M + 4 * r, ge[0], ge[1], ge[2], ge[3]);
                }
                __syncthreads();  // (1) partials written
                {
                    const int q = t >> 6, i = t & 63;
                    float z = 0.f;
#pragma unroll
                    for (int rr = 0; rr < 16; ++rr) z += sm.red[q][rr][i];
                    sm.fin[q][i] = z;
                }
                __syncthreads();  // (2) totals
                // gbeta = u.h - u.Ru, the same sum in every warp
                float gbt;
                {
                    const int l = t & 31;
                    float z = sm.hu[x][2 * l] * sm.fin[1][2 * l] + sm.hu[x][2 * l + 1] * sm.fin[1][2 * l + 1];
                    if (l < 16) z -= sm.urup[par][l];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
                    gbt = z;
                }
                const float gs = (s >= floor_) ? -beta * beta * gbt : 0.f;
                float gu_r[4], gu_c[4];
                {
                    float h_r[4], h_c[4], rr_r[4], rr_c[4];
                    unpack(ld4(sm.fin[1] + 4 * r), h_r);
                    unpack(ld4(sm.fin[1] + 4 * c), h_c);
                    unpack(ld4(sm.ru[par] + 4 * r), rr_r);
                    unpack(ld4(sm.ru[par] + 4 * c), rr_c);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        gu_r[i] = fmaf(gs, k_r[i], beta * h_r[i] - 2.f * beta * rr_r[i]);
                        gu_c[i] = fmaf(gs, k_c[i], beta * h_c[i] - 2.f * beta * rr_c[i]);
                    }
                }
                // gk = -A (Mp ge) + gs u + Pbar gu; S = R + sym(gu k^T);
                // ga = gMbar . Mp + 2 (S o Pp) a; R <- A S A
                float pgk[4], pga[4], tr = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    float zk = 0.f, za = 0.f;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float aa = a_r[i] * a_c[j];
                        float pb = aa * Pp[i][j];
                        if (r == c && i == j) pb += p;
                        zk = fmaf(pb, gu_c[j], zk);
                        const float S = R[i][j] + 0.5f * (__fmul_rn(gu_r[i], k_c[j]) + __fmul_rn(gu_c[j], k_r[i]));
                        za = fmaf(S * Pp[i][j], a_c[j], za);
                        if (r == c && i == j) tr += S;
                        R[i][j] = aa * S;
                    }
                    pgk[i] = zk;
                    pga[i] = za;
                }
                // key and decay gradients at row 4r + ((c >> 2) & 3), one lane of each group of four
                const float gkv = hw_scatter4(pgk), gav = hw_scatter4(pga);
                if (r == c) sm.trp[x][r] = tr;
                if ((c & 3) == 0) {
                    const int ri = (c >> 2) & 3, kr = 4 * r + ri;
                    A.gk[row * D + kr] = gkv + gs * pick(u_r, ri) - pick(a_r, ri) * sm.fin[2][kr];
                    if (NEED_DYN) A.ga[row * D + kr] = FIXED ? 0.f : fmaf(2.f, gav, sm.fin[3][kr]);
                }
                if (c == 0) {
                    float gq4[4];
                    unpack(ld4(sm.fin[0] + 4 * r), gq4);
                    st4(A.gq + row * D + 4 * r, gq4[0], gq4[1], gq4[2], gq4[3]);
                }
                if (NEED_DYN && t == 0) A.gr[row] = FIXED ? 0.f : gs;
            }
            __syncthreads();  // traces complete
            if (NEED_DYN && t < slen) {
                float z = 0.f;
#pragma unroll
                for (int q = 0; q < 16; ++q) z += sm.trp[t][q];
                A.gp[chain * T + t0 + s0 + t] = FIXED ? 0.f : z;
            }
        }
    }
    if (NEED_INIT) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            st4(A.gm0 + chain * D * M + (4 * c + i) * M + 4 * r, gM[i][0], gM[i][1], gM[i][2], gM[i][3]);
            st4(A.gc0 + chain * D * D + (4 * r + i) * D + 4 * c, R[i][0], R[i][1], R[i][2], R[i][3]);
        }
    }
}

template <bool FIXED, bool DYN, bool INIT>
int launch_bwd(const BwdArgs<float> &a, cudaStream_t st) {
    auto k = d64_backward<FIXED, DYN, INIT>;
    static const bool attr =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sizeof(BwdSmem))) ==
        cudaSuccess;
    if (!attr) return fail(BSSM_ERR_CUDA, "d64 backward: shared-memory attribute refused");
    k<<<static_cast<unsigned>(a.n), kThreads, sizeof(BwdSmem), st>>>(a);
    return check_launch("d64 backward");
}

}  // namespace d64

size_t d64_workspace_bytes(long n, long t, int chunks) {
    if (n <= 0 || t <= 0 || chunks <= 0) return 0;
    const long span = chunks < t ? chunks : t;
    const long nsub = (span + d64::kSub - 1) / d64::kSub;
    if (nsub <= 1) return 0;
    return static_cast<size_t>(n) * static_cast<size_t>(nsub - 1) * d64::kStateFloats * sizeof(float);
}

int d64_forward(int fixed, const FwdArgs<float> &a, cudaStream_t st) {
    if (a.n > 0x7fffffffL) return fail(BSSM_ERR_INVALID, "d64: too many chains");
    if (a.out == nullptr && a.t > 0) return fail(BSSM_ERR_INVALID, "d64 forward: null output");
    const unsigned grid = static_cast<unsigned>(a.n);
    if (fixed) {
        d64::d64_forward<true><<<grid, d64::kThreads, 0, st>>>(a);
    } else {
        d64::d64_forward<false><<<grid, d64::kThreads, 0, st>>>(a);
    }
    return check_launch("d64 forward");
}

int d64_backward(int fixed, bool dyn, bool init, const BwdArgs<float> &a, cudaStream_t st) {
    if (a.n > 0x7fffffffL) return fail(BSSM_ERR_INVALID, "d64: too many chains");
    if (a.ws == nullptr && d64_workspace_bytes(a.n, a.t, a.chunks) > 0)
        return fail(BSSM_ERR_WORKSPACE, "d64 backward: workspace required");
    const int key = (fixed ? 4 : 0) | (dyn ? 2 : 0) | (init ? 1 : 0);
    switch (key) {
        case 0: return d64::launch_bwd<false, false, false>(a, st);
        case 1: return d64::launch_bwd<false, false, true>(a, st);
        case 2: return d64::launch_bwd<false, true, false>(a, st);
        case 3: return d64::launch_bwd<false, true, true>(a, st);
        case 4: return d64::launch_bwd<true, false, false>(a, st);
        case 5: return d64::launch_bwd<true, false, true>(a, st);
        case 6: return d64::launch_bwd<true, true, false>(a, st);
        default: return d64::launch_bwd<true, true, true>(a, st);
    }
}

}  // namespace bssm
