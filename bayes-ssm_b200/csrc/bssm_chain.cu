// bssm_chain.cu -- thread-per-chain forward and replay backward for sm_100a.
//
// Same recurrence and adjoint as the other kernel families (catid/bayes-ssm
// bayes_ssm/bayesian_layer.py:153-181 and :207-251; adjoint formula sheet
// bayes_ssm/persistent_bayes_chunked_d8.cu:358-419), organised so that one
// thread owns one chain:
//
// * The thread keeps the chain's covariance as its upper triangle (D(D+1)/2
//   registers) and its mean as D x M registers.  The predict / update /
//   readout and the whole reverse step are thread-local: no shuffle, no
//   partial sums to exchange, and every symmetric covariance entry (and its
//   adjoint) is computed once.
// * A CTA is 4 warps = 128 chains; a warp's 32 chains are consecutive.  Token
//   inputs move by TMA: per tile of kS tokens, one lane issues one tensor copy
//   per input field for the warp's 32 chains.  The tensor maps traverse
//   (row, chain, token), so a tile lands token-major in shared memory and
//   thread c reads its row of token tau at [tau][c][.]: consecutive threads,
//   consecutive rows, no bank conflict and no per-thread address arithmetic.
//   Outputs leave the same way (staged rows, then TMA tensor stores).
// * Backward (one launch): for each kS-token sub-chunk, last to first, the
//   thread reloads the sub-chunk's start state (saved by the forward every kS
//   tokens, or the boundary checkpoint), replays the sub-chunk -- a
//   covariance pass, then a mean pass -- and runs the reverse step over it.
//   The per-token history (pre-step mean and covariance, gain, innovation,
//   beta, s) lives in tensor memory: lane = chain, ~120 columns per token at
//   D8M8.  Registers hold only the adjoint state (dL/dM, R = sym dL/dP) and
//   the working set of one token.
//
// The TMA path needs tile starts and rows aligned to 16 bytes: T and the
// chunk length multiples of kS, key rows of 16 bytes (D8 in BF16, D4/D8 in
// FP32).  chain_eligible() checks this; other shapes use the other families.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "bayes_ssm_b200.h"
#include "bssm_common.cuh"
#include "bssm_internal.h"
#include "bssm_tmem.cuh"

namespace bssm {
namespace chain {

constexpr int kS = kReplaySpan;  // tokens per tile = replay sub-chunk
constexpr int kWarps = 4;        // one warp per TMEM lane quarter
constexpr int kThreads = 32 * kWarps;
constexpr int kSplitWarps = 8;  // two warps per chain group
constexpr int kSplitThreads = 32 * kSplitWarps;
constexpr int kSmemMax = 227 * 1024;

// Unroll factors of the per-token loops of the two-warp (split) kernels.
// Measured at config 3 (16,384 chains, T 512, one B200): unrolling the
// backward's two replay loops fully took it from 0.867 to 0.824 ms; fully
// unrolled adjoint loops were slower (0.965 ms; 1.18 ms together with the
// replays), 2-way neutral; the forward's loops were neutral at 2 and slower
// at 4 (0.432 -> 0.472 ms).  Also neutral (within 0.5 %): loading the
// covariance warp's tile rows before its exchange wait, splitting its
// gain-adjoint sum into two chains, and the replay update in packed pairs.
#ifndef BSSM_SPLIT_UNROLL_FWD
#define BSSM_SPLIT_UNROLL_FWD 1
#endif
#ifndef BSSM_SPLIT_UNROLL_REPLAY
#define BSSM_SPLIT_UNROLL_REPLAY 4
#endif
#ifndef BSSM_SPLIT_UNROLL_COV
#define BSSM_SPLIT_UNROLL_COV 1
#endif
#ifndef BSSM_SPLIT_UNROLL_MEAN
#define BSSM_SPLIT_UNROLL_MEAN 1
#endif
constexpr int kUnrollFwd = BSSM_SPLIT_UNROLL_FWD;        // forward_split, both warps
constexpr int kUnrollReplay = BSSM_SPLIT_UNROLL_REPLAY;  // backward_split replays
constexpr int kUnrollCov = BSSM_SPLIT_UNROLL_COV;        // backward_split covariance adjoint
constexpr int kUnrollMean = BSSM_SPLIT_UNROLL_MEAN;      // backward_split mean adjoint

constexpr int al128(int x) { return (x + 127) / 128 * 128; }
constexpr int al1024(int x) { return (x + 1023) / 1024 * 1024; }
// Start of a region of line boxes whose lines span `span` bytes: swizzled
// lines (32 bytes and up) need the swizzle atom's 1024-byte alignment;
// 16-byte lines are not swizzled and need only the TMA's 128 bytes.
constexpr int al_line(int x, int span) { return span == 16 ? al128(x) : al1024(x); }
// Shared memory one CTA may take when two share an SM (228 KB per SM, 1 KB
// reserved per CTA).
constexpr int kSmemTwoPerSm = (228 * 1024 - 2 * 1024) / 2;

// N consecutive floats from 16-byte aligned shared memory.
template <int N>
__device__ __forceinline__ void lds_n(const float *p, float (&o)[N]) {
#pragma unroll
    for (int i = 0; i + 4 <= N; i += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(p + i);
        o[i] = v.x; o[i + 1] = v.y; o[i + 2] = v.z; o[i + 3] = v.w;
    }
    constexpr int b = N / 4 * 4;
    if constexpr (N % 4 >= 2) {
        const float2 v = *reinterpret_cast<const float2 *>(p + b);
        o[b] = v.x; o[b + 1] = v.y;
    }
    if constexpr (N % 2 == 1) o[N - 1] = p[N - 1];
}
__device__ __forceinline__ float sel4(const float (&x)[4], int i) {
    return i == 0 ? x[0] : i == 1 ? x[1] : i == 2 ? x[2] : x[3];
}


__device__ __forceinline__ float sel4v(const float4 &x, int i) {
    return i == 0 ? x.x : i == 1 ? x.y : i == 2 ? x.z : x.w;
}

// ---- packed FP32 pairs (sm_100 f32x2 arithmetic) -----------------------------
// Row-major D x M means pair up along the value dimension: pr(x, c) is
// (x[c], x[c+1]).  One f32x2 instruction does the two lanes' IEEE operations,
// so a loop over value pairs computes exactly what the scalar loop over
// values would, in half the instructions.
__device__ __forceinline__ float2 bc2(float s) { return make_float2(s, s); }
__device__ __forceinline__ float2 pr(const float *x, int c) { return make_float2(x[c], x[c + 1]); }
__device__ __forceinline__ void spr(float *x, int c, float2 v) {
    x[c] = v.x;
    x[c + 1] = v.y;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
// sum_c x[c] y[c] over M (even) values: pairwise partial sums, then one add
template <int M>
__device__ __forceinline__ float dot2(const float *x, const float *y) {
    static_assert(M % 2 == 0, "value pairs");
    float2 acc = mul2(pr(x, 0), pr(y, 0));
#pragma unroll
    for (int c = 2; c < M; c += 2) acc = fma2(pr(x, c), pr(y, c), acc);
    return acc.x + acc.y;
}
// y[c] = sum_i X[i][c] w[i] for every value c (value pairs, i in order)
template <int D, int M>
__device__ __forceinline__ void colsum2(const float (&X)[D][M], const float (&w)[D], float (&y)[M]) {
    static_assert(M % 2 == 0, "value pairs");
#pragma unroll
    for (int c = 0; c < M; c += 2) {
        float2 acc = mul2(pr(X[0], c), bc2(w[0]));
#pragma unroll
        for (int i = 1; i < D; ++i) acc = fma2(pr(X[i], c), bc2(w[i]), acc);
        spr(y, c, acc);
    }
}
// dL/dM' += q gy^T
template <int D, int M>
__device__ __forceinline__ void add_outer2(float (&gM)[D][M], const float (&qv)[D], const float (&gy)[M]) {
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int c = 0; c < M; c += 2) spr(gM[i], c, fma2(bc2(qv[i]), pr(gy, c), pr(gM[i], c)));
}
// acc = gM^T u; ge = beta acc (the value gradient); returns e . acc (= u^T gM e)
template <int D, int M>
__device__ __forceinline__ float gain_adjoint2(const float (&gM)[D][M], const float (&u)[D], const float (&e)[M],
                                               float beta, float (&ge)[M]) {
    float acc[M];
    colsum2<D, M>(gM, u, acc);
#pragma unroll
    for (int c = 0; c < M; c += 2) spr(ge, c, mul2(bc2(beta), pr(acc, c)));
    return dot2<M>(e, acc);
}
// One row i of the mean adjoint through the update, given the pre-step mean
// row mp: pk = mp . ge; g = gM_i - k_i ge; ga = g . mp (with DYN); gM_i = a_i g.
template <int M, bool DYN>
__device__ __forceinline__ void mean_row_adjoint2(float (&gmi)[M], const float (&mp)[M], const float (&ge)[M],
                                                  float k, float a, float &pk, float &ga) {
    static_assert(M % 2 == 0, "value pairs");
    const float2 nk = bc2(-k), a2 = bc2(a);
    float2 g = fma2(nk, pr(ge, 0), pr(gmi, 0));
    float2 pacc = mul2(pr(mp, 0), pr(ge, 0)), gacc = mul2(g, pr(mp, 0));
    spr(gmi, 0, mul2(a2, g));
#pragma unroll
    for (int c = 2; c < M; c += 2) {
        pacc = fma2(pr(mp, c), pr(ge, c), pacc);
        g = fma2(nk, pr(ge, c), pr(gmi, c));
        if constexpr (DYN) gacc = fma2(g, pr(mp, c), gacc);
        spr(gmi, c, mul2(a2, g));
    }
    pk = pacc.x + pacc.y;
    ga = DYN ? gacc.x + gacc.y : 0.f;
}

// ---- mbarriers ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint64_t *bar, int bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
// Bounded wait for the phase of the given parity.  A wait that gives up is
// counted in a device word (the kernel then runs on with wrong results
// instead of hanging); bssm_stream_status() turns a new count into
// BSSM_ERR_TIMEOUT, and the Python layer raises on it after every call.
__device__ unsigned int g_wait_timeouts = 0;
constexpr int kWaitLimit = 1 << 22;
__device__ __forceinline__ bool mbar_wait_n(uint64_t *bar, uint32_t parity, int limit) {
    const uint32_t addr = smem_u32(bar);
    for (int it = 0; it < limit; ++it) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
    }
    atomicAdd(&g_wait_timeouts, 1u);
    return false;
}
__device__ __forceinline__ void mbar_wait(uint64_t *bar, uint32_t parity) { mbar_wait_n(bar, parity, kWaitLimit); }

// Diagnostic: one thread waits, with `limit` polls, on a barrier phase that
// nothing completes, so the bounded wait gives up and is counted exactly as
// a give-up inside a recurrence kernel would be.
__global__ void wait_probe_kernel(int limit) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_init_fence();
        mbar_wait_n(&bar, 0, limit);
    }
}

// ---- TMA tensor copies (this CTA's shared memory only) ----------------------
__device__ __forceinline__ void tma_load_2d(void *sdst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(sdst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int x, int y, const void *ssrc) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_u32(ssrc))
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// at most N of the issuing thread's committed groups may still read shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Tensor maps of one launch.  Token maps traverse (row x token, chain) with a
// line box of (kS rows, 32 chains); noise maps (token, chain) with a box of
// (kS tokens, 32 chains); the replay-state map (float, chain) with a box of
// (one state, 32 chains).
struct FwdMaps {
    CUtensorMap k, q, v, a, p, r, y, gu, gb;  // gu, gb: gains and signed gain scales
    int gains;  // the one-warp forward saves the gains (only the two-warp backward reads them)
};
struct BwdMaps {
    CUtensorMap k, q, v, a, p, r, gy, rs, gk, gv, gq, ga, gp, gr, gu, gb;
};

// ---- Line layout -------------------------------------------------------------
// Token tensors [N, T, row] travel as line boxes: for each of 32 consecutive
// chains, the kS rows of tokens [t0, t0 + kS) form one line of
// L = kS * rowbytes bytes (16, 32, 64 or 128), contiguous in global memory,
// so TMA moves one segment per chain.  TMA writes (and reads back) a box with
// the swizzle of span L: the 16-byte chunk x of chain c's line sits at chunk
// x ^ s(c), with s(c) = (c >> 2) & 1, (c >> 1) & 3 and c & 7 for L = 32, 64
// and 128 (bits [4, ..) of the offset in a 1024-byte aligned region XOR bits
// [7, ..)); 16-byte lines are not swizzled.  A warp's 16-byte accesses to one
// chunk of its 32 chains then fall in distinct banks within each quarter warp.
template <int L>
__device__ __forceinline__ int line_chunk(int c, int x) {
    static_assert(L == 16 || L == 32 || L == 64 || L == 128, "line span");
    if constexpr (L == 16) {
        return c * 16;
    } else if constexpr (L == 32) {
        return c * 32 + ((x ^ ((c >> 2) & 1)) << 4);
    } else if constexpr (L == 64) {
        return c * 64 + ((x ^ ((c >> 1) & 3)) << 4);
    } else {
        return c * 128 + ((x ^ (c & 7)) << 4);
    }
}

// One 16-byte chunk: 4 floats, or 8 floats rounded to BF16.
__device__ __forceinline__ void sts_chunk(float *p, const float *x) {
    *reinterpret_cast<float4 *>(p) = make_float4(x[0], x[1], x[2], x[3]);
}
__device__ __forceinline__ void sts_chunk(__nv_bfloat16 *p, const float *x) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t *>(&h);
    }
    *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ uint32_t word_of(const uint4 &w, int i) {
    return i == 0 ? w.x : i == 1 ? w.y : i == 2 ? w.z : w.w;
}

// Row tau (N elements of T) of chain c, from or to a line region.  Rows of
// 16 bytes or more are whole chunks; shorter rows (4 or 8 bytes) are words of
// one chunk.
template <int N, typename T>
__device__ __forceinline__ void line_load(const char *region, int c, int tau, float (&o)[N]) {
    constexpr int RB = N * static_cast<int>(sizeof(T)), L = kS * RB, EC = 16 / static_cast<int>(sizeof(T));
    static_assert(RB % 4 == 0, "rows of whole words");
    if constexpr (RB >= 16) {
#pragma unroll
        for (int h = 0; h < RB / 16; ++h) {
            float x[EC];
            lds_vec<EC>(reinterpret_cast<const T *>(region + line_chunk<L>(c, tau * (RB / 16) + h)), x);
#pragma unroll
            for (int e = 0; e < EC; ++e) o[h * EC + e] = x[e];
        }
    } else {
        const int byte = tau * RB;
        const uint4 w = *reinterpret_cast<const uint4 *>(region + line_chunk<L>(c, byte >> 4));
        const int w0 = (byte & 15) >> 2;
#pragma unroll
        for (int i = 0; i < RB / 4; ++i) {
            const uint32_t x = word_of(w, w0 + i);
            if constexpr (sizeof(T) == 4) {
                o[i] = __uint_as_float(x);
            } else {
                o[2 * i] = bf16_lo(x);
                o[2 * i + 1] = bf16_hi(x);
            }
        }
    }
}
template <int N, typename T>
__device__ __forceinline__ void line_store(char *region, int c, int tau, const float (&v)[N]) {
    constexpr int RB = N * static_cast<int>(sizeof(T)), L = kS * RB, EC = 16 / static_cast<int>(sizeof(T));
    static_assert(RB % 4 == 0, "rows of whole words");
    if constexpr (RB >= 16) {
#pragma unroll
        for (int h = 0; h < RB / 16; ++h)
            sts_chunk(reinterpret_cast<T *>(region + line_chunk<L>(c, tau * (RB / 16) + h)), v + h * EC);
    } else {
        uint32_t x[RB / 4];
#pragma unroll
        for (int i = 0; i < RB / 4; ++i) {
            if constexpr (sizeof(T) == 4) {
                x[i] = __float_as_uint(v[i]);
            } else {
                const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                x[i] = *reinterpret_cast<const uint32_t *>(&h);
            }
        }
        const int byte = tau * RB;
        char *const dst = region + line_chunk<L>(c, byte >> 4) + (byte & 15);
        if constexpr (RB == 4) {
            *reinterpret_cast<uint32_t *>(dst) = x[0];
        } else {
            *reinterpret_cast<uint2 *>(dst) = make_uint2(x[0], x[1]);
        }
    }
}

// A lane's replay state as float quads: quad x at +128 x floats, both in the
// global state part (from replay_state_base) and in a group's state box
// [SF / 4][32 chains][4] (from box + 4 lane).
template <int D, int M>
struct StateQuads {
    static constexpr int SF = replay_state_floats(D, M), DM = D * M, TRI = tri_size(D);
    static_assert(DM % 4 == 0, "mean in whole quads");
    __device__ __forceinline__ static void put_mean(float *dst, const float (&Mm)[D][M]) {
#pragma unroll
        for (int f = 0; f < DM; f += 4)
            *reinterpret_cast<float4 *>(dst + f * 32) =
                make_float4(Mm[f / M][f % M], Mm[(f + 1) / M][(f + 1) % M], Mm[(f + 2) / M][(f + 2) % M],
                            Mm[(f + 3) / M][(f + 3) % M]);
    }
    __device__ __forceinline__ static void put_cov(float *dst, const float (&P)[TRI]) {
#pragma unroll
        for (int f = 0; f < SF - DM; f += 4) {
            float x[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) x[e] = f + e < TRI ? P[f + e] : 0.f;
            *reinterpret_cast<float4 *>(dst + (DM + f) * 32) = make_float4(x[0], x[1], x[2], x[3]);
        }
    }
    __device__ __forceinline__ static void get_mean(const float *src, float (&Mm)[D][M]) {
#pragma unroll
        for (int f = 0; f < DM; f += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(src + f * 32);
            Mm[f / M][f % M] = v.x;
            Mm[(f + 1) / M][(f + 1) % M] = v.y;
            Mm[(f + 2) / M][(f + 2) % M] = v.z;
            Mm[(f + 3) / M][(f + 3) % M] = v.w;
        }
    }
    __device__ __forceinline__ static void get_cov(const float *src, float (&P)[TRI]) {
#pragma unroll
        for (int f = 0; f < SF - DM; f += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(src + (DM + f) * 32);
            const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (f + e < TRI) P[f + e] = x[e];
        }
    }
};

// Shared-memory geometry of one warp's tile (one stage): line boxes of the
// token tensors, [chain][tau] boxes of the noise.
template <int D, int M, bool FIXED, bool BWD, typename TIn>
struct Tile {
    static constexpr int rbK = D * static_cast<int>(sizeof(TIn)), rbV = M * static_cast<int>(sizeof(TIn));
    static constexpr int szK = kS * 32 * rbK, szV = kS * 32 * rbV, szA = FIXED ? 0 : kS * 32 * D * 4;
    static constexpr int szP = FIXED ? 0 : 32 * kS * 4, szG = BWD ? kS * 32 * M * 4 : 0;
    // line regions, aligned for their swizzle, then the [chain][tau] noise
    // rows; the tile itself spans whole KB so every warp's tile starts
    // 1024-byte aligned
    static constexpr int spK = kS * rbK, spV = kS * rbV, spA = kS * D * 4, spG = kS * M * 4;
    static constexpr int oK = 0, oQ = al_line(oK + szK, spK), oV = al_line(oQ + szK, spV);
    static constexpr int oA = al_line(oV + szV, spA), oG = al_line(oA + szA, spG), oP = al128(oG + szG);
    static constexpr int oR = oP + szP;
    static constexpr int kBytes = al1024(oR + szP);
    static constexpr int kTx = 2 * szK + szV + szA + 2 * szP;  // bytes the token maps deliver, without gy
};

// The warp's copies of tokens [t0, t0+kS) of chains [chain0, chain0+32),
// issued by one lane; the stage is complete when `bytes` have landed.
template <int D, int M, bool FIXED, bool BWD, typename TIn, typename Maps>
__device__ __forceinline__ void issue_tile(char *tile, const Maps &mp, int chain0, int t0, bool with_gy,
                                           uint64_t *bar, int extra_bytes) {
    using Tl = Tile<D, M, FIXED, BWD, TIn>;
    mbar_arrive_tx(bar, Tl::kTx + (with_gy ? Tl::szG : 0) + extra_bytes);
    tma_load_2d(tile + Tl::oK, &mp.k, t0 * D, chain0, bar);
    tma_load_2d(tile + Tl::oQ, &mp.q, t0 * D, chain0, bar);
    tma_load_2d(tile + Tl::oV, &mp.v, t0 * M, chain0, bar);
    if constexpr (!FIXED) {
        tma_load_2d(tile + Tl::oA, &mp.a, t0 * D, chain0, bar);
        tma_load_2d(tile + Tl::oP, &mp.p, t0, chain0, bar);
        tma_load_2d(tile + Tl::oR, &mp.r, t0, chain0, bar);
    }
    if constexpr (BWD) {
        if (with_gy) tma_load_2d(tile + Tl::oG, &mp.gy, t0 * M, chain0, bar);
    }
}

// Reads of token tau's rows for lane c from a tile.
template <int D, int M, bool FIXED, bool BWD, typename TIn>
struct TileRead {
    using Tl = Tile<D, M, FIXED, BWD, TIn>;
    const char *t;
    int c;
    __device__ __forceinline__ void keys(int tau, float (&k)[D]) const {
        line_load<D, TIn>(t + Tl::oK, c, tau, k);
    }
    __device__ __forceinline__ void queries(int tau, float (&q)[D]) const {
        line_load<D, TIn>(t + Tl::oQ, c, tau, q);
    }
    __device__ __forceinline__ void values(int tau, float (&v)[M]) const {
        line_load<M, TIn>(t + Tl::oV, c, tau, v);
    }
    __device__ __forceinline__ void decay(int tau, float (&a)[D]) const {
        if constexpr (FIXED) {
#pragma unroll
            for (int j = 0; j < D; ++j) a[j] = kFixedDecay;
        } else {
            line_load<D, float>(t + Tl::oA, c, tau, a);
        }
    }
    __device__ __forceinline__ void noise(float4 &p4, float4 &r4) const {
        if constexpr (FIXED) {
            p4 = make_float4(kFixedProcess, kFixedProcess, kFixedProcess, kFixedProcess);
            r4 = make_float4(kFixedObservation, kFixedObservation, kFixedObservation, kFixedObservation);
        } else {
            p4 = reinterpret_cast<const float4 *>(t + Tl::oP)[c];
            r4 = reinterpret_cast<const float4 *>(t + Tl::oR)[c];
        }
    }
    __device__ __forceinline__ void gy(int tau, float (&g)[M]) const {
        line_load<M, float>(t + Tl::oG, c, tau, g);
    }
};

// ---------------------------------------------------------------------------
// The recurrence on one thread's registers.  P is the packed upper triangle.
// Products are the same commutative pairs, in the same order, as the other
// kernel families use.
// ---------------------------------------------------------------------------
template <int D>
__device__ __forceinline__ void cov_step(float (&P)[tri_size(D)], const float (&k)[D], const float (&a)[D],
                                         float p, float r, float floor_, float (&u)[D], float &beta, float &s) {
    float wk[D];
#pragma unroll
    for (int j = 0; j < D; ++j) wk[j] = a[j] * k[j];
#pragma unroll
    for (int i = 0; i < D; ++i) {
        float z = 0.f;
#pragma unroll
        for (int j = 0; j < D; ++j) z = fmaf(P[tri_index(D, i, j)], wk[j], z);
        u[i] = fmaf(a[i], z, p * k[i]);
    }
    s = r;
#pragma unroll
    for (int j = 0; j < D; ++j) s = fmaf(k[j], u[j], s);
    // clamp_min (NaN stays NaN), then the fast reciprocal: 2 ulp, well inside
    // the FP32 parity bar, and it shortens the covariance warp's serial
    // chain; the saved gain scale carries this same value to the backward
    beta = __fdividef(1.0f, s < floor_ ? floor_ : s);
    float nbu[D];
#pragma unroll
    for (int i = 0; i < D; ++i) nbu[i] = -beta * u[i];
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int j = i; j < D; ++j) {
            const int t = tri_index(D, i, j);
            const float upd = fmaf(nbu[i], u[j], (a[i] * a[j]) * P[t]);
            P[t] = (i == j) ? upd + p : upd;
        }
}

// e = v - (A M)^T k and M' = A M + beta u e^T, in value pairs.
template <int D, int M>
__device__ __forceinline__ void mean_step(float (&Mm)[D][M], const float (&k)[D], const float (&a)[D],
                                          const float (&v)[M], const float (&u)[D], float beta, float (&e)[M]) {
    static_assert(M % 2 == 0, "value pairs");
    float nwk[D];
#pragma unroll
    for (int i = 0; i < D; ++i) nwk[i] = -(a[i] * k[i]);
#pragma unroll
    for (int c = 0; c < M; c += 2) {
        float2 acc = mul2(pr(Mm[0], c), bc2(nwk[0]));
#pragma unroll
        for (int i = 1; i < D; ++i) acc = fma2(pr(Mm[i], c), bc2(nwk[i]), acc);
        spr(e, c, add2(pr(v, c), acc));
    }
#pragma unroll
    for (int c = 0; c < M; c += 2) {
        const float2 be = mul2(bc2(beta), pr(e, c));
#pragma unroll
        for (int i = 0; i < D; ++i) spr(Mm[i], c, fma2(bc2(a[i]), pr(Mm[i], c), mul2(be, bc2(u[i]))));
    }
}

// State <-> global memory (row-major mean, full covariance).
template <int D, int M>
__device__ __forceinline__ void store_mean(float *dst, const float (&Mm)[D][M]) {
#pragma unroll
    for (int i = 0; i < D; ++i) store_vec<M>(dst + i * M, Mm[i]);
}
template <int D>
__device__ __forceinline__ void store_cov_full(float *dst, const float (&P)[tri_size(D)]) {
#pragma unroll
    for (int i = 0; i < D; ++i) {
        float row[D];
#pragma unroll
        for (int j = 0; j < D; ++j) row[j] = P[tri_index(D, i, j)];
        store_vec<D>(dst + i * D, row);
    }
}
// Order in which a chain's tiles are consumed by the forward: chunk by chunk,
// kS-token sub-chunks in order (sub-chunks restart at every chunk boundary,
// so the replay states sit at tile starts).
struct FwdItems {
    long T, ci, nb;
    int L, j, nsub, len;
    bool done;
    __device__ __forceinline__ void enter() {
        const long t0 = ci * L;
        len = static_cast<int>((T - t0) < L ? (T - t0) : L);
        nsub = (len + kS - 1) / kS;
        j = 0;
    }
    __device__ __forceinline__ void init(long T_, int L_) {
        T = T_;
        L = L_;
        nb = (T + L - 1) / L;
        ci = 0;
        done = nb <= 0;
        if (!done) enter();
    }
    __device__ __forceinline__ void advance() {
        if (++j >= nsub) {
            if (++ci >= nb) {
                done = true;
            } else {
                enter();
            }
        }
    }
    __device__ __forceinline__ long t0() const { return ci * L + static_cast<long>(j) * kS; }
    __device__ __forceinline__ int ntok() const { return (len - j * kS) < kS ? (len - j * kS) : kS; }
};

template <int D, int M, bool FIXED, typename TIn>
struct FwdGeo {
    using Tl = Tile<D, M, FIXED, false, TIn>;
    static constexpr int SF = replay_state_floats(D, M);
    // a warp's outputs of one tile: readout and gains as line boxes, the
    // signed gain scales [chain][tau]
    static constexpr int yY = 0, yU = al1024(kS * 32 * M * 4), yB = yU + kS * 32 * D * 4;
    static constexpr int kYB = al1024(yB + 32 * kS * 4);
    static constexpr int kPerStage = kWarps * Tl::kBytes;
    static constexpr int kFixed = kWarps * kYB + 1024 + kWarps * 4 * 8;
    static constexpr int kFit = (kSmemMax - kFixed) / kPerStage;
    static constexpr bool kFits = kFit >= 2;  // else the shape goes to another family
    // Two CTAs per SM when two or more stages still fit in half the SM's
    // shared memory (small rows: at D2 a lone CTA left three warps of every
    // four sub-partition slots empty and ran 65,536 chains in four waves),
    // else up to four stages in one CTA.
    static constexpr int kFitTwo = (kSmemTwoPerSm - kFixed - kWarps * 4 * 8 - 1024) / kPerStage;
    static constexpr int kStages = kFitTwo >= 2 ? (kFitTwo < 4 ? kFitTwo : 4) : (kFit < 2 ? 2 : (kFit < 4 ? kFit : 4));
    static constexpr int oY = 0;                            // [warp][kYB]
    static constexpr int oT = oY + kWarps * kYB;            // [stage][warp][tile]
    static constexpr int oBar = oT + kStages * kPerStage;   // [warp][stage]
    static constexpr int kSmem = oBar + kWarps * kStages * 8 + 1024;  // + alignment slack
    static_assert(!kFits || kSmem <= kSmemMax, "forward shared memory");
};

// 1024-byte aligned start of dynamic shared memory (swizzled line boxes).
__device__ __forceinline__ char *smem_base(char *raw) {
    const uint32_t a = smem_u32(raw);
    return raw + ((1024 - (a & 1023)) & 1023);
}

// ===========================================================================
// Forward
// ===========================================================================
template <int D, int M, bool FIXED, typename TIn>
__global__ void __launch_bounds__(kThreads, 1) forward_chain(const FwdArgs<TIn> A, const __grid_constant__ FwdMaps mp) {
    using G = FwdGeo<D, M, FIXED, TIn>;
    using Tl = typename G::Tl;
    constexpr int NS = G::kStages, TRI = tri_size(D), SF = G::SF;
    extern __shared__ __align__(128) char smem_raw[];
    char *const smem = smem_base(smem_raw);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int chain0 = static_cast<int>(blockIdx.x) * kThreads + warp * 32;
    const long chain = chain0 + lane;
    const bool active = chain < A.n;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;
    const long rs_slots = replay_slots_per_chunk(T, L);
    char *const tiles = smem + G::oT + warp * Tl::kBytes;  // + stage * G::kPerStage
    char *const ob = smem + G::oY + warp * G::kYB;
    uint64_t *const bars = reinterpret_cast<uint64_t *>(smem + G::oBar) + warp * NS;
    if (lane == 0) {
        for (int s = 0; s < NS; ++s) mbar_init(bars + s, 1);
        mbar_init_fence();
    }
    __syncwarp();

    float Mm[D][M], P[TRI];
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int c = 0; c < M; ++c) Mm[i][c] = 0.f;
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int j = i; j < D; ++j) P[tri_index(D, i, j)] = (i == j) ? 1.f : 0.f;
    if (active && A.mean0 != nullptr) {
#pragma unroll
        for (int i = 0; i < D; ++i) load_vec<M>(A.mean0 + chain * D * M + i * M, Mm[i]);
    }
    if (active && A.cov0 != nullptr) {
        const float *c0 = A.cov0 + chain * D * D;
#pragma unroll
        for (int i = 0; i < D; ++i)
#pragma unroll
            for (int j = i; j < D; ++j) P[tri_index(D, i, j)] = 0.5f * (c0[i * D + j] + c0[j * D + i]);
    }
    float *const bm = A.bmean + chain * (nb + 1) * D * M;
    float *const bc = A.bcov + chain * (nb + 1) * D * D;

    FwdItems prod, cons;
    prod.init(T, L);
    cons.init(T, L);
    if (lane == 0) {
        for (int s = 0; s < NS - 1 && !prod.done; ++s) {
            issue_tile<D, M, FIXED, false, TIn>(tiles + s * G::kPerStage, mp, chain0, static_cast<int>(prod.t0()),
                                                false, bars + s, 0);
            prod.advance();
        }
    } else {
        for (int s = 0; s < NS - 1 && !prod.done; ++s) prod.advance();
    }
    long q = 0;
    while (!cons.done) {
        // every lane is done with the stage about to be refilled (it held tile q-1)
        __syncwarp();
        if (!prod.done) {
            const int st = static_cast<int>((q + NS - 1) % NS);
            if (lane == 0)
                issue_tile<D, M, FIXED, false, TIn>(tiles + st * G::kPerStage, mp, chain0,
                                                    static_cast<int>(prod.t0()), false, bars + st, 0);
            prod.advance();
        }
        mbar_wait(bars + q % NS, static_cast<uint32_t>((q / NS) & 1));
        const TileRead<D, M, FIXED, false, TIn> rd{tiles + (q % NS) * G::kPerStage, lane};
        const long ci = cons.ci;
        const int t0 = static_cast<int>(cons.t0());
        if (cons.j == 0) {
            if (active) {
                store_mean<D, M>(bm + ci * D * M, Mm);
                store_cov_full<D>(bc + ci * D * D, P);
            }
        }
        if (cons.j != 0 && A.rs != nullptr && active) {
            // the state, quad by quad: each store of the warp is one
            // contiguous 512-byte line of the state part
            float *const dst = A.rs + replay_state_base(chain, nb, rs_slots, ci, cons.j, SF);
            StateQuads<D, M>::put_mean(dst, Mm);
            StateQuads<D, M>::put_cov(dst, P);
        }
        char *const yb = ob + G::yY;
        const bool gains = A.rs != nullptr && mp.gains != 0;
        float4 p4, r4, b4 = make_float4(0.f, 0.f, 0.f, 0.f);
        rd.noise(p4, r4);
        auto step = [&](int tau) {
            float k[D], a[D], v[M], qv[D];
            const float p = sel4v(p4, tau), r = sel4v(r4, tau);
            rd.keys(tau, k);
            rd.decay(tau, a);
            rd.values(tau, v);
            float u[D], e[M], beta, s;
            cov_step<D>(P, k, a, p, r, A.floor, u, beta, s);
            mean_step<D, M>(Mm, k, a, v, u, beta, e);
            rd.queries(tau, qv);
            float y[M];
            colsum2<D, M>(Mm, qv, y);
            if (tau == 0) {
                // the output staging was last read by tile q-1's output stores
                if (lane == 0) bulk_wait_read<0>();
                __syncwarp();
            }
            line_store<M, float>(yb, lane, tau, y);
            if (gains) {
                line_store<D, float>(ob + G::yU, lane, tau, u);
                const float bt = signed_gain_scale(beta, s, A.floor);
                b4.x = tau == 0 ? bt : b4.x;
                b4.y = tau == 1 ? bt : b4.y;
                b4.z = tau == 2 ? bt : b4.z;
                b4.w = tau == 3 ? bt : b4.w;
            }
        };
#pragma unroll 1
        for (int tau = 0; tau < kS; ++tau) step(tau);
        if (gains) reinterpret_cast<float4 *>(ob + G::yB)[lane] = b4;
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
            if (chain0 < A.n) {
                tma_store_2d(&mp.y, t0 * M, chain0, yb);
                if (gains) {
                    tma_store_2d(&mp.gu, t0 * D, chain0, ob + G::yU);
                    tma_store_2d(&mp.gb, t0, chain0, ob + G::yB);
                }
            }
            bulk_commit();
        }
        cons.advance();
        ++q;
    }
    if (active) {
        store_mean<D, M>(bm + nb * D * M, Mm);
        store_cov_full<D>(bc + nb * D * D, P);
        store_mean<D, M>(A.mean_final + chain * D * M, Mm);
        store_cov_full<D>(A.cov_final + chain * D * D, P);
    }
    if (lane == 0) bulk_wait_all();
}

// ===========================================================================
// Forward with two warps per chain group (D = M = 8)
//
// Group g's covariance warp (warp g) runs the covariance recursion -- P, u,
// s, beta -- and writes the gains of each tile into a double-buffered
// shared-memory block; the mean warp (warp g + 4) reads them there and runs
// the mean recursion and the readout, one tile behind.  Both warps store
// their half of each replay state directly (structure-of-arrays rows), the
// covariance warp stores the gains (TMA), the mean warp the readout (TMA,
// staged in the tile's own decay slots once they are dead).
// ===========================================================================
template <int D, int M, bool FIXED, typename TIn>
struct FSplitGeo {
    using Tl = Tile<D, M, FIXED, false, TIn>;
    static constexpr bool kInPlaceY = !FIXED && D == M;  // readout rows fit the decay slots
    static constexpr int gU = 0, gB = kS * 32 * D * 4;
    static constexpr int kGB = al1024(gB + 32 * kS * 4);   // one gains block: u (line box), signed scale
    static constexpr int kYB = kInPlaceY ? 0 : kS * 32 * M * 4;
    static constexpr int kPerStage = 4 * Tl::kBytes;
    static constexpr int kBars = 2 * 4 + 4;                // full[4] empty[4] gfull[2] gfree[2]
    static constexpr int kFixed = 4 * (2 * kGB + kYB) + 4 * kBars * 8 + 1024 + 128;
    static constexpr int kFit = (kSmemMax - kFixed) / kPerStage;
    static constexpr int kStages = kFit < 4 ? kFit : 4;
    static constexpr bool kFits = kStages >= 3;
    static constexpr int oT = 0;                                      // [stage][group][tile]
    static constexpr int oG = kStages * kPerStage;                    // [group][2][kGB]
    static constexpr int oY = oG + 4 * 2 * kGB;                       // [group][kYB]
    static constexpr int oBar = al128(oY + 4 * kYB);                  // [group][kBars]
    static constexpr int kSmem = oBar + 4 * kBars * 8 + 1024;  // + alignment slack
};

template <int D, int M, bool FIXED, typename TIn>
__global__ void __launch_bounds__(kSplitThreads, 1)
    forward_split(const FwdArgs<TIn> A, const __grid_constant__ FwdMaps mp) {
    using G = FSplitGeo<D, M, FIXED, TIn>;
    using Tl = typename G::Tl;
    constexpr int NS = G::kStages, TRI = tri_size(D), SF = replay_state_floats(D, M);
    extern __shared__ __align__(128) char smem_raw[];
    char *const smem = smem_base(smem_raw);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int grp = warp & 3;
    const bool cov_warp = warp < 4;
    const int chain0 = static_cast<int>(blockIdx.x) * 128 + grp * 32;
    const long chain = chain0 + lane;
    const bool active = chain < A.n;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;
    const long rs_slots = replay_slots_per_chunk(T, L);
    char *const tiles = smem + G::oT + grp * Tl::kBytes;  // + stage * G::kPerStage
    char *const gbuf = smem + G::oG + grp * 2 * G::kGB;   // + b * G::kGB
    uint64_t *const bars = reinterpret_cast<uint64_t *>(smem + G::oBar) + grp * G::kBars;
    uint64_t *const full = bars, *const empty = bars + 4, *const gfull = bars + 8, *const gfree = bars + 10;
    float *const bm = A.bmean + chain * (nb + 1) * D * M;
    float *const bc = A.bcov + chain * (nb + 1) * D * D;
    const bool gains_out = A.rs != nullptr;

    if (cov_warp && lane == 0) {
        for (int x = 0; x < 4; ++x) {
            mbar_init(full + x, 1);
            mbar_init(empty + x, 2);
        }
        for (int x = 0; x < 2; ++x) {
            mbar_init(gfull + x, 32);
            mbar_init(gfree + x, 32);
        }
        mbar_init_fence();
    }
    __syncthreads();

    FwdItems cons;
    cons.init(T, L);
    if (cov_warp) {
        // ------------------------------------------------------------------
        // covariance warp; its lane 0 also issues the tiles
        // ------------------------------------------------------------------
        float P[TRI];
#pragma unroll
        for (int i = 0; i < D; ++i)
#pragma unroll
            for (int j = i; j < D; ++j) P[tri_index(D, i, j)] = (i == j) ? 1.f : 0.f;
        if (active && A.cov0 != nullptr) {
            const float *c0 = A.cov0 + chain * D * D;
#pragma unroll
            for (int i = 0; i < D; ++i)
#pragma unroll
                for (int j = i; j < D; ++j) P[tri_index(D, i, j)] = 0.5f * (c0[i * D + j] + c0[j * D + i]);
        }
        // tiles run NS - 2 ahead: the stage a new tile goes to held the tile
        // two before the current one, which the mean warp released
        FwdItems prod = cons;
        if (lane == 0) {
            for (int s = 0; s < NS - 2 && !prod.done; ++s) {
                issue_tile<D, M, FIXED, false, TIn>(tiles + s * G::kPerStage, mp, chain0, static_cast<int>(prod.t0()),
                                                    false, full + s, 0);
                prod.advance();
            }
        } else {
            for (int s = 0; s < NS - 2 && !prod.done; ++s) prod.advance();
        }
        long q = 0;
        while (!cons.done) {
            if (!prod.done) {
                const long nq = q + NS - 2;
                if (lane == 0) {
                    if (nq >= NS) mbar_wait(empty + nq % NS, static_cast<uint32_t>(((nq - NS) / NS) & 1));
                    issue_tile<D, M, FIXED, false, TIn>(tiles + (nq % NS) * G::kPerStage, mp, chain0,
                                                        static_cast<int>(prod.t0()), false, full + nq % NS, 0);
                }
                prod.advance();
            }
            mbar_wait(full + q % NS, static_cast<uint32_t>((q / NS) & 1));
            const TileRead<D, M, FIXED, false, TIn> rd{tiles + (q % NS) * G::kPerStage, lane};
            const long ci = cons.ci;
            const int t0 = static_cast<int>(cons.t0());
            if (active) {
                if (cons.j == 0) {
                    store_cov_full<D>(bc + ci * D * D, P);
                } else if (A.rs != nullptr) {
                    StateQuads<D, M>::put_cov(A.rs + replay_state_base(chain, nb, rs_slots, ci, cons.j, SF), P);
                }
            }
            // gains block q & 1: free once the mean warp read tile q-2's gains
            // and this warp's store of them read its source
            const int b = static_cast<int>(q & 1);
            char *const gb = gbuf + b * G::kGB;
            if (q >= 2) mbar_wait(gfree + b, static_cast<uint32_t>(((q - 2) >> 1) & 1));
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
            float4 p4, r4, b4 = make_float4(0.f, 0.f, 0.f, 0.f);
            rd.noise(p4, r4);
#pragma unroll kUnrollFwd
            for (int tau = 0; tau < kS; ++tau) {
                float k[D], a[D], u[D], beta, s;
                rd.keys(tau, k);
                rd.decay(tau, a);
                cov_step<D>(P, k, a, sel4v(p4, tau), sel4v(r4, tau), A.floor, u, beta, s);
                line_store<D, float>(gb + G::gU, lane, tau, u);
                const float bt = signed_gain_scale(beta, s, A.floor);
                b4.x = tau == 0 ? bt : b4.x;
                b4.y = tau == 1 ? bt : b4.y;
                b4.z = tau == 2 ? bt : b4.z;
                b4.w = tau == 3 ? bt : b4.w;
            }
            reinterpret_cast<float4 *>(gb + G::gB)[lane] = b4;
            fence_proxy_async();
            mbar_arrive(gfull + b);
            __syncwarp();
            if (lane == 0) {
                if (gains_out && chain0 < A.n) {
                    tma_store_2d(&mp.gu, t0 * D, chain0, gb + G::gU);
                    tma_store_2d(&mp.gb, t0, chain0, gb + G::gB);
                }
                bulk_commit();
                mbar_arrive(empty + q % NS);  // this warp is done with the tile
            }
            cons.advance();
            ++q;
        }
        if (active) {
            store_cov_full<D>(bc + nb * D * D, P);
            store_cov_full<D>(A.cov_final + chain * D * D, P);
        }
    } else {
        // ------------------------------------------------------------------
        // mean warp
        // ------------------------------------------------------------------
        float Mm[D][M];
#pragma unroll
        for (int i = 0; i < D; ++i)
#pragma unroll
            for (int c = 0; c < M; ++c) Mm[i][c] = 0.f;
        if (active && A.mean0 != nullptr) {
#pragma unroll
            for (int i = 0; i < D; ++i) load_vec<M>(A.mean0 + chain * D * M + i * M, Mm[i]);
        }
        char *const ysep = smem + G::oY + grp * G::kYB;
        long q = 0;
        while (!cons.done) {
            if constexpr (G::kInPlaceY) {
                // the previous tile's readout store has read its decay slots:
                // release that stage before waiting for this tile
                if (lane == 0 && q >= 1) {
                    bulk_wait_read<0>();
                    mbar_arrive(empty + (q - 1) % NS);
                }
            }
            mbar_wait(full + q % NS, static_cast<uint32_t>((q / NS) & 1));
            const int b = static_cast<int>(q & 1);
            mbar_wait(gfull + b, static_cast<uint32_t>((q >> 1) & 1));
            char *const tile = tiles + (q % NS) * G::kPerStage;
            const TileRead<D, M, FIXED, false, TIn> rd{tile, lane};
            const char *const gb = gbuf + b * G::kGB;
            const long ci = cons.ci;
            const int t0 = static_cast<int>(cons.t0());
            if (active) {
                if (cons.j == 0) {
                    store_mean<D, M>(bm + ci * D * M, Mm);
                } else if (A.rs != nullptr) {
                    StateQuads<D, M>::put_mean(A.rs + replay_state_base(chain, nb, rs_slots, ci, cons.j, SF), Mm);
                }
            }
            char *yb;
            if constexpr (G::kInPlaceY) {
                yb = tile + Tl::oA;  // decay rows die token by token
            } else {
                yb = ysep;
                if (lane == 0) bulk_wait_read<0>();  // the previous readout store
                __syncwarp();
            }
            const float4 b4 = reinterpret_cast<const float4 *>(gb + G::gB)[lane];
#pragma unroll kUnrollFwd
            for (int tau = 0; tau < kS; ++tau) {
                float k[D], a[D], v[M], qv[D], u[D], e[M];
                rd.keys(tau, k);
                rd.decay(tau, a);
                rd.values(tau, v);
                line_load<D, float>(gb + G::gU, lane, tau, u);
                mean_step<D, M>(Mm, k, a, v, u, fabsf(sel4v(b4, tau)), e);
                rd.queries(tau, qv);
                float y[M];
                colsum2<D, M>(Mm, qv, y);
                line_store<M, float>(yb, lane, tau, y);
            }
            mbar_arrive(gfree + b);  // done with this gains block
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                if (chain0 < A.n) tma_store_2d(&mp.y, t0 * M, chain0, yb);
                bulk_commit();
                if constexpr (!G::kInPlaceY) mbar_arrive(empty + q % NS);
            }
            cons.advance();
            ++q;
        }
        if (active) {
            store_mean<D, M>(bm + nb * D * M, Mm);
            store_mean<D, M>(A.mean_final + chain * D * M, Mm);
        }
    }
    if (lane == 0) bulk_wait_all();
}

// ===========================================================================
// Backward
// ===========================================================================

// TMEM columns of one lane (= one chain).  Fields, each kept for the kS
// tokens of the current sub-chunk:
// (kRp, one copy: the covariance adjoint, parked while the sub-chunk is
// replayed so that its registers serve the replay.)
enum Field { kMp = 0, kPp = 1, kU = 2, kE = 3, kBS = 4, kRp = 5, kNumFields = 6 };
// Every field is split into power-of-two pieces of at most 32 columns
// (binary expansion, largest first); all pieces of one width are placed
// together, widest first, so every piece starts at a multiple of its width.
template <int D, int M>
struct TLayout {
    __host__ __device__ static constexpr int size(int f) {
        return f == kMp ? D * M : f == kPp ? tri_size(D) : f == kU ? D : f == kE ? M : f == kBS ? 2 : tri_size(D);
    }
    __host__ __device__ static constexpr int copies(int f) { return f == kRp ? 1 : kS; }
    __host__ __device__ static constexpr int npieces(int n, int w) { return w == 32 ? n / 32 : (((n % 32) & w) ? 1 : 0); }
    // position inside the field of the first piece of width w
    __host__ __device__ static constexpr int piece_pos(int n, int w) {
        int p = (n / 32) * 32;
        if (w == 32) return 0;
        for (int x = 16; x > w; x >>= 1)
            if ((n % 32) & x) p += x;
        return p;
    }
    // column of the first piece of width w of field f, token 0
    __host__ __device__ static constexpr int col0(int f, int w) {
        int c = 0;
        for (int x = 32; x > w; x >>= 1)
            for (int g = 0; g < kNumFields; ++g) c += copies(g) * npieces(size(g), x) * x;
        for (int g = 0; g < f; ++g) c += copies(g) * npieces(size(g), w) * w;
        return c;
    }
    __host__ __device__ static constexpr int total() {
        int c = 0;
        for (int x = 32; x >= 1; x >>= 1)
            for (int g = 0; g < kNumFields; ++g) c += copies(g) * npieces(size(g), x) * x;
        return c;
    }
    __host__ __device__ static constexpr int alloc() {
        int a = 32;
        while (a < total()) a *= 2;
        return a;
    }
    static_assert(total() <= 512, "history does not fit in tensor memory");
};

template <class TL, int F, int W = 32>
__device__ __forceinline__ void field_st(uint32_t base, int tau, const uint32_t *r) {
    constexpr int n = TL::size(F), np = TL::npieces(n, W);
    if constexpr (np > 0) {
        constexpr int c0 = TL::col0(F, W), pos = TL::piece_pos(n, W);
#pragma unroll
        for (int idx = 0; idx < np; ++idx) tmem::st_cols<W>(base + c0 + (tau * np + idx) * W, r + pos + idx * W);
    }
    if constexpr (W > 1) field_st<TL, F, W / 2>(base, tau, r);
}
template <class TL, int F, int W = 32>
__device__ __forceinline__ void field_ld(uint32_t base, int tau, uint32_t *r) {
    constexpr int n = TL::size(F), np = TL::npieces(n, W);
    if constexpr (np > 0) {
        constexpr int c0 = TL::col0(F, W), pos = TL::piece_pos(n, W);
#pragma unroll
        for (int idx = 0; idx < np; ++idx) tmem::ld_cols<W>(base + c0 + (tau * np + idx) * W, r + pos + idx * W);
    }
    if constexpr (W > 1) field_ld<TL, F, W / 2>(base, tau, r);
}
// Store N floats as field F of token (or slot) tau.
template <class TL, int F, int N>
__device__ __forceinline__ void put(uint32_t base, int tau, const float *v) {
    static_assert(N == TL::size(F), "field size");
    uint32_t r[N];
#pragma unroll
    for (int i = 0; i < N; ++i) r[i] = __float_as_uint(v[i]);
    field_st<TL, F>(base, tau, r);
}
// Load field F of token (or slot) tau (waits for the load).
template <class TL, int F, int N>
__device__ __forceinline__ void get(uint32_t base, int tau, float *v) {
    static_assert(N == TL::size(F), "field size");
    uint32_t r[N];
    field_ld<TL, F>(base, tau, r);
    tmem::wait_ld_bind<N>(r);
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = __uint_as_float(r[i]);
}
// Load rows [R0, R0+NR) of the pre-step mean (field FM) of token tau.  The
// mean field is row-major, so for M = 8 a 32-column piece is 4 whole rows.
template <class TL, int FM, int D, int M, int R0, int NR>
__device__ __forceinline__ void get_mean_rows(uint32_t base, int tau, float (&out)[NR][M]) {
    constexpr int n = D * M;
    uint32_t r[NR * M];
    if constexpr (n >= 32) {
        static_assert((R0 * M) % 32 == 0 && (NR * M) % 32 == 0, "row block = whole pieces");
        constexpr int np = TL::npieces(n, 32), c0 = TL::col0(FM, 32);
#pragma unroll
        for (int b = 0; b < NR * M / 32; ++b)
            tmem::ld_cols<32>(base + c0 + (tau * np + R0 * M / 32 + b) * 32, r + 32 * b);
    } else {
        static_assert(R0 == 0 && NR == D, "small means load whole");
        field_ld<TL, FM>(base, tau, r);
    }
    tmem::wait_ld_bind<NR * M>(r);
#pragma unroll
    for (int i = 0; i < NR; ++i)
#pragma unroll
        for (int c = 0; c < M; ++c) out[i][c] = __uint_as_float(r[i * M + c]);
}

// Consumption order of the backward: chunks from the last, kS-token
// sub-chunks from the last.
struct BwdItems {
    long T, ci;
    int L, j, nsub, len;
    bool done;
    __device__ __forceinline__ void enter() {
        const long t0 = ci * L;
        len = static_cast<int>((T - t0) < L ? (T - t0) : L);
        nsub = (len + kS - 1) / kS;
        j = nsub - 1;
    }
    __device__ __forceinline__ void init(long T_, int L_) {
        T = T_;
        L = L_;
        ci = (T + L - 1) / L - 1;
        done = ci < 0;
        if (!done) enter();
    }
    __device__ __forceinline__ void advance() {
        if (--j < 0) {
            if (--ci < 0) {
                done = true;
            } else {
                enter();
            }
        }
    }
    __device__ __forceinline__ long t0() const { return ci * L + static_cast<long>(j) * kS; }
    __device__ __forceinline__ int ntok() const { return (len - j * kS) < kS ? (len - j * kS) : kS; }
};


template <int D, int M, bool FIXED, typename TIn>
struct BwdGeo {
    using Tl = Tile<D, M, FIXED, true, TIn>;
    static constexpr int SF = replay_state_floats(D, M);
    static constexpr int kSB = 32 * SF * 4;  // a warp's start states, box layout [SF / 4][chain][4]
    // a warp's gradient rows of one sub-chunk: keys, values, queries, decay
    // as line boxes (whole KB each); process, observation [chain][tau]
    static constexpr int rbK = Tl::rbK, rbV = Tl::rbV;
    static constexpr int gK = 0, gV = al_line(gK + kS * 32 * rbK, Tl::spV), gQ = al_line(gV + kS * 32 * rbV, Tl::spK);
    static constexpr int gA = al_line(gQ + kS * 32 * rbK, Tl::spA), gP = al128(gA + kS * 32 * D * 4);
    static constexpr int gR = gP + 32 * kS * 4, kOB = al1024(gR + 32 * kS * 4);
    static constexpr int kPerStage = kWarps * Tl::kBytes;
    static constexpr int oT = 0;                              // [stage][warp][tile]
    static constexpr int oS = oT + 2 * kPerStage;             // [warp][kSB]
    static constexpr int oO = al1024(oS + kWarps * kSB);      // [warp][kOB]
    static constexpr bool kStageOut = oO + kWarps * kOB + kWarps * 2 * 8 + 16 + 1024 <= kSmemMax;
    static constexpr int oBar = kStageOut ? oO + kWarps * kOB : oO;  // [warp][stage]
    static constexpr int oSlot = oBar + kWarps * 2 * 8;
    static constexpr int kSmem = oSlot + 16 + 1024;  // + alignment slack
    static_assert(kSmem <= kSmemMax, "backward shared memory");
};

// One gradient row of token tau: into the staging line box (written back at
// the sub-chunk's end), or straight to global memory.
template <bool STAGE, int N, typename T>
__device__ __forceinline__ void put_row(char *region, int c, int tau, T *gdst, const float (&v)[N], bool active) {
    if constexpr (STAGE) {
        line_store<N, T>(region, c, tau, v);
    } else if (active) {
        store_vec<N>(gdst, v);
    }
}

// Copy a sub-chunk's start state from a boundary checkpoint (full
// covariance, by its upper triangle) into this thread's state row.
// (The state box is [SF / 4][32 chains][4]: this thread's float f at
// sdst + 4 rs_at(0, f).)
template <int D, int M>
__device__ __forceinline__ void issue_checkpoint(uint32_t sdst, const float *ck_mean, const float *ck_cov) {
#pragma unroll
    for (int x = 0; x < D * M; ++x) cp_async<4>(sdst + 4 * rs_at(0, x), ck_mean + x);
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int j = i; j < D; ++j)
            cp_async<4>(sdst + 4 * rs_at(0, D * M + tri_index(D, i, j)), ck_cov + i * D + j);
}

// First row of a group's state (ci, j) in the [rows][32 chains x 4] view of
// the quad-interleaved state part.
__device__ __forceinline__ int state_row(int chain0, long nb, long slots, long ci, long j, int sf) {
    return static_cast<int>((((static_cast<long>(chain0) >> 5) * nb + ci) * slots + (j - 1)) * (sf / 4));
}

template <int D, int M, bool FIXED, bool NEED_DYN, bool NEED_INIT, typename TIn>
__global__ void __launch_bounds__(kThreads, 1) backward_chain(const BwdArgs<TIn> A, const __grid_constant__ BwdMaps mp) {
    using G = BwdGeo<D, M, FIXED, TIn>;
    using Tl = typename G::Tl;
    using TL = TLayout<D, M>;
    constexpr int TRI = tri_size(D), SF = G::SF;
    extern __shared__ __align__(128) char smem_raw[];
    char *const smem = smem_base(smem_raw);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int chain0 = static_cast<int>(blockIdx.x) * kThreads + warp * 32;
    const long chain = chain0 + lane;
    const bool active = chain < A.n;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;
    const long rs_slots = replay_slots_per_chunk(T, L);
    const float floor_ = A.floor;
    const bool has_gy = A.gy != nullptr;
    char *const tiles = smem + G::oT + warp * Tl::kBytes;  // + stage * G::kPerStage
    float *const sbox = reinterpret_cast<float *>(smem + G::oS + warp * G::kSB);  // [SF][32 chains]
    float *const state = sbox + 4 * lane;                                         // quads at +128 x
    char *const out = smem + G::oO + warp * G::kOB;
    uint64_t *const bars = reinterpret_cast<uint64_t *>(smem + G::oBar) + warp * 2;
    uint32_t *const slot = reinterpret_cast<uint32_t *>(smem + G::oSlot);
    const float *const bm = A.bmean + chain * (nb + 1) * D * M;
    const float *const bc = A.bcov + chain * (nb + 1) * D * D;

    for (int x = 0; x < SF; ++x) state[rs_at(0, x)] = 0.f;  // idle lanes replay finite zeros
    if (lane == 0) {
        mbar_init(bars, 1);
        mbar_init(bars + 1, 1);
        mbar_init_fence();
    }
    if (warp == 0) {
        tmem::alloc(slot, TL::alloc());
        tmem::relinquish();
    }
    tmem::fence_before_sync();
    __syncthreads();
    tmem::fence_after_sync();
    // this warp's lane quarter; the thread's own lane is implicit
    const uint32_t tb = *slot + (static_cast<uint32_t>(warp * 32) << 16);

    // adjoint state: dL/d(mean) and R = sym(dL/d(covariance)), packed
    float gM[D][M], Rp[TRI];
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int c = 0; c < M; ++c) gM[i][c] = 0.f;
#pragma unroll
    for (int t = 0; t < TRI; ++t) Rp[t] = 0.f;
    if (active && A.gmf != nullptr) {
#pragma unroll
        for (int i = 0; i < D; ++i) load_vec<M>(A.gmf + chain * D * M + i * M, gM[i]);
    }
    if (active && A.gcf != nullptr) {
        const float *gc = A.gcf + chain * D * D;
#pragma unroll
        for (int i = 0; i < D; ++i)
#pragma unroll
            for (int j = i; j < D; ++j) Rp[tri_index(D, i, j)] = 0.5f * (gc[i * D + j] + gc[j * D + i]);
    }

    // one item: the sub-chunk's input tile and its start state (a saved
    // replay state in the same TMA transaction, or a boundary checkpoint by
    // per-thread copies)
    auto issue_item = [&](const BwdItems &it, int stage) {
        const bool saved = it.j > 0;
        if (lane == 0) {
            uint64_t *bar = bars + stage;
            issue_tile<D, M, FIXED, true, TIn>(tiles + stage * G::kPerStage, mp, chain0, static_cast<int>(it.t0()),
                                               has_gy, bar, saved ? G::kSB : 0);
            if (saved) tma_load_2d(sbox, &mp.rs, 0, state_row(chain0, nb, rs_slots, it.ci, it.j, SF), bar);
        }
        if (!saved && active) issue_checkpoint<D, M>(smem_u32(state), bm + it.ci * D * M, bc + it.ci * D * D);
        cp_async_commit();
    };

    BwdItems prod, cons;
    prod.init(T, L);
    cons.init(T, L);
    if (!prod.done) {
        issue_item(prod, 0);
        prod.advance();
    }
    long q = 0;
    while (!cons.done) {
        cp_async_wait<0>();
        mbar_wait(bars + (q & 1), static_cast<uint32_t>((q >> 1) & 1));
        const TileRead<D, M, FIXED, true, TIn> rd{tiles + (q & 1) * G::kPerStage, lane};
        const int t0 = static_cast<int>(cons.t0());
        const long row0 = chain * T + t0;
        float4 p4, r4;
        rd.noise(p4, r4);
        put<TLayout<D, M>, kRp, TRI>(tb, 0, Rp);  // parked during the replay

        // ---- covariance pass: pre-step covariance, gain, beta and s per token
        {
            float P[TRI];
            StateQuads<D, M>::get_cov(state, P);
            auto cstep = [&](int tau) {
                float k[D], a[D], u[D], bs[2];
                rd.keys(tau, k);
                rd.decay(tau, a);
                put<TLayout<D, M>, kPp, TRI>(tb, tau, P);
                cov_step<D>(P, k, a, sel4v(p4, tau), sel4v(r4, tau), floor_, u, bs[0], bs[1]);
                put<TLayout<D, M>, kU, D>(tb, tau, u);
                put<TLayout<D, M>, kBS, 2>(tb, tau, bs);
            };
#pragma unroll 1
            for (int tau = 0; tau < kS; ++tau) cstep(tau);
        }
        tmem::wait_st();
        // ---- mean pass: pre-step mean and innovation per token; gq = M' gy
        {
            float Mm[D][M];
            StateQuads<D, M>::get_mean(state, Mm);
            // every lane has read its start state and is done with the other
            // stage: fetch the next sub-chunk while this one is processed.
            // The next start state lands in the same box by TMA (async proxy);
            // the proxy fence orders this lane's reads of the box before it.
            // Without it a read still queued could see the next state: at two
            // CTAs per SM that made the key-dim-2 gradients differ run to run.
            fence_proxy_async();
            __syncwarp();
            if (!prod.done) {
                issue_item(prod, static_cast<int>((q + 1) & 1));
                prod.advance();
            }
            if constexpr (G::kStageOut) {
                if (lane == 0) bulk_wait_read<0>();  // the previous sub-chunk's gradient stores
                __syncwarp();
            }
            auto mstep = [&](int tau) {
                float k[D], a[D], v[M], u[D], bs[2], e[M];
                rd.keys(tau, k);
                rd.decay(tau, a);
                rd.values(tau, v);
                get<TLayout<D, M>, kU, D>(tb, tau, u);
                get<TLayout<D, M>, kBS, 2>(tb, tau, bs);
                {
                    float flat[D * M];
#pragma unroll
                    for (int i = 0; i < D; ++i)
#pragma unroll
                        for (int c = 0; c < M; ++c) flat[i * M + c] = Mm[i][c];
                    put<TLayout<D, M>, kMp, D * M>(tb, tau, flat);
                }
                mean_step<D, M>(Mm, k, a, v, u, bs[0], e);
                put<TLayout<D, M>, kE, M>(tb, tau, e);
                float gq[D];
                if (has_gy) {
                    float gy[M];
                    rd.gy(tau, gy);
#pragma unroll
                    for (int i = 0; i < D; ++i) gq[i] = dot2<M>(Mm[i], gy);
                } else {
#pragma unroll
                    for (int i = 0; i < D; ++i) gq[i] = 0.f;
                }
                put_row<G::kStageOut, D>(out + G::gQ, lane, tau, A.gq + (row0 + tau) * D, gq, active);
            };
#pragma unroll 1
            for (int tau = 0; tau < kS; ++tau) mstep(tau);
        }
        tmem::wait_st();
        get<TLayout<D, M>, kRp, TRI>(tb, 0, Rp);

        // ---- reverse step over the sub-chunk
        float4 gp4 = make_float4(0.f, 0.f, 0.f, 0.f), gr4 = gp4;
        auto rstep = [&](int tau) {
            const long row = row0 + tau;
            float k[D], a[D];
            const float p = sel4v(p4, tau);
            rd.keys(tau, k);
            rd.decay(tau, a);
            float u[D], e[M], bs[2];
            get<TLayout<D, M>, kU, D>(tb, tau, u);
            get<TLayout<D, M>, kE, M>(tb, tau, e);
            get<TLayout<D, M>, kBS, 2>(tb, tau, bs);
            const float beta = bs[0], s = bs[1];
            // dL/d(post-update mean)
            if (has_gy) {
                float qv[D], gy[M];
                rd.queries(tau, qv);
                rd.gy(tau, gy);
                add_outer2<D, M>(gM, qv, gy);
            }
            float ge[M], h[D];
            float gb = gain_adjoint2<D, M>(gM, u, e, beta, ge);  // u^T gM' e
#pragma unroll
            for (int i = 0; i < D; ++i) h[i] = dot2<M>(gM[i], e);
            // pre-step mean: -A M ge (keys), decay gradient, dL/d(pre-step mean)
            float pk[D], gam[D];
            constexpr int RB = (D * M >= 32) ? 32 / M : D;  // rows per TMEM load
#pragma unroll
            for (int r0 = 0; r0 < D; r0 += RB) {
                float Mp[RB][M];
                if constexpr (RB == D) {
                    get_mean_rows<TLayout<D, M>, kMp, D, M, 0, D>(tb, tau, Mp);
                } else {
                    if (r0 == 0) {
                        get_mean_rows<TLayout<D, M>, kMp, D, M, 0, RB>(tb, tau, Mp);
                    } else {
                        get_mean_rows<TLayout<D, M>, kMp, D, M, RB, RB>(tb, tau, Mp);
                    }
                }
#pragma unroll
                for (int ii = 0; ii < RB; ++ii) {
                    const int i = r0 + ii;
                    mean_row_adjoint2<M, NEED_DYN>(gM[i], Mp[ii], ge, k[i], a[i], pk[i], gam[i]);
                }
            }
            // covariance adjoint
            float Ru[D], trR = 0.f;
#pragma unroll
            for (int i = 0; i < D; ++i) {
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) acc = fmaf(Rp[tri_index(D, i, j)], u[j], acc);
                Ru[i] = acc;
                gb = fmaf(-u[i], acc, gb);
                if constexpr (NEED_DYN) trR += Rp[tri_index(D, i, i)];
            }
            const float gs = (s >= floor_) ? -beta * beta * gb : 0.f;
            float gu[D], ag[D];
#pragma unroll
            for (int i = 0; i < D; ++i) {
                gu[i] = beta * h[i] - 2.f * beta * Ru[i] + gs * k[i];
                ag[i] = a[i] * gu[i];
            }
            float Pp[TRI];
            get<TLayout<D, M>, kPp, TRI>(tb, tau, Pp);
            float gk[D];
#pragma unroll
            for (int i = 0; i < D; ++i) {
                float z = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) z = fmaf(Pp[tri_index(D, i, j)], ag[j], z);
                const float gk3 = fmaf(a[i], z, p * gu[i]);
                gk[i] = fmaf(-a[i], pk[i], fmaf(gs, u[i], gk3));
            }
            float gaP[D];
            float hg[D];  // gu / 2
#pragma unroll
            for (int i = 0; i < D; ++i) {
                gaP[i] = 0.f;
                hg[i] = 0.5f * gu[i];
            }
#pragma unroll
            for (int i = 0; i < D; ++i)
#pragma unroll
                for (int j = i; j < D; ++j) {
                    const int t = tri_index(D, i, j);
                    // S = R + sym(gu k^T), upper triangle
                    const float S = i == j ? fmaf(gu[i], k[i], Rp[t]) : fmaf(hg[i], k[j], fmaf(hg[j], k[i], Rp[t]));
                    if constexpr (NEED_DYN) {
                        const float w = S * Pp[t];
                        gaP[i] = fmaf(w, a[j], gaP[i]);
                        if (i != j) gaP[j] = fmaf(w, a[i], gaP[j]);
                    }
                    Rp[t] = (a[i] * a[j]) * S;
                }
            put_row<G::kStageOut, D>(out + G::gK, lane, tau, A.gk + row * D, gk, active);
            put_row<G::kStageOut, M>(out + G::gV, lane, tau, A.gv + row * M, ge, active);
            if constexpr (NEED_DYN) {
                float ga[D], gpv, grv;
                if constexpr (FIXED) {
#pragma unroll
                    for (int i = 0; i < D; ++i) ga[i] = 0.f;
                    gpv = 0.f;
                    grv = 0.f;
                } else {
                    float gpk = 0.f;
#pragma unroll
                    for (int i = 0; i < D; ++i) {
                        ga[i] = fmaf(2.f, gaP[i], gam[i]);
                        gpk = fmaf(gu[i], k[i], gpk);
                    }
                    gpv = trR + gpk;
                    grv = gs;
                }
                put_row<G::kStageOut, D>(out + G::gA, lane, tau, A.ga + row * D, ga, active);
                if constexpr (G::kStageOut) {
                    gp4.x = tau == 0 ? gpv : gp4.x;
                    gp4.y = tau == 1 ? gpv : gp4.y;
                    gp4.z = tau == 2 ? gpv : gp4.z;
                    gp4.w = tau == 3 ? gpv : gp4.w;
                    gr4.x = tau == 0 ? grv : gr4.x;
                    gr4.y = tau == 1 ? grv : gr4.y;
                    gr4.z = tau == 2 ? grv : gr4.z;
                    gr4.w = tau == 3 ? grv : gr4.w;
                } else if (active) {
                    A.gp[row] = gpv;
                    A.gr[row] = grv;
                }
            }
        };
#pragma unroll 1
        for (int tau = kS - 1; tau >= 0; --tau) rstep(tau);
        if constexpr (G::kStageOut) {
            if constexpr (NEED_DYN) {
                reinterpret_cast<float4 *>(out + G::gP)[lane] = gp4;
                reinterpret_cast<float4 *>(out + G::gR)[lane] = gr4;
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0 && chain0 < A.n) {
                tma_store_2d(&mp.gk, t0 * D, chain0, out + G::gK);
                tma_store_2d(&mp.gv, t0 * M, chain0, out + G::gV);
                tma_store_2d(&mp.gq, t0 * D, chain0, out + G::gQ);
                if constexpr (NEED_DYN) {
                    tma_store_2d(&mp.ga, t0 * D, chain0, out + G::gA);
                    tma_store_2d(&mp.gp, t0, chain0, out + G::gP);
                    tma_store_2d(&mp.gr, t0, chain0, out + G::gR);
                }
                bulk_commit();
            }
        }
        cons.advance();
        ++q;
    }
    cp_async_wait<0>();
    if constexpr (NEED_INIT) {
        if (active) {
            store_mean<D, M>(A.gm0 + chain * D * M, gM);
            store_cov_full<D>(A.gc0 + chain * D * D, Rp);
        }
    }
    if constexpr (G::kStageOut) {
        if (lane == 0) bulk_wait_all();
    }
    tmem::fence_before_sync();
    __syncthreads();
    tmem::fence_after_sync();
    if (warp == 0) tmem::dealloc(*slot, TL::alloc());
}

// ===========================================================================
// Backward with two warps per chain group (D = M, BF16 inputs, dynamic
// noise): the headline configuration.
//
// Group g (32 chains) has a covariance warp (warp g) and a mean warp (warp
// g + 4).  Both sit on SM sub-partition g and reach TMEM lane quarter g, so
// they share the chains' tensor-memory lanes; the sub-partition interleaves
// two instruction streams instead of one.
//   covariance warp: replays the covariance from the gains the forward saved
//     (history: pre-step covariance), then runs the R-adjoint of the reverse
//     step;
//   mean warp: replays the mean from the same gains (history: pre-step mean,
//     innovation), writes gq, then runs the dL/dM adjoint and hands the
//     covariance warp, per token, h = gM' e, pk = M ge, the decay term of the
//     mean and u.gM'.e through a ring of three TMEM slots.
// With the gains saved the two replays are independent; the warps meet only
// at the exchange ring and at the tile stages.  Synchronisation is by
// mbarriers (tile stage full / free, start state read, exchange slot full /
// free).  The gradient rows are staged in the tile's own input slots once
// those inputs are dead (gk in keys, gv in queries, gq in values, ga in
// decay, gp in process, gr in observation) and leave by TMA stores.
// ===========================================================================
constexpr int kXSlots = 3;

// TMEM columns of one lane in the two-warp backward.
enum SplitField { kSMp = 0, kSPp = 1, kSE = 2, kSX = 3, kSNumFields = 4 };
template <int D, int M>
struct TLayoutSplit {
    __host__ __device__ static constexpr int size(int f) {
        return f == kSMp ? D * M : f == kSPp ? tri_size(D) : f == kSE ? M : 3 * D + 1;
    }
    __host__ __device__ static constexpr int copies(int f) { return f == kSX ? kXSlots : kS; }
    __host__ __device__ static constexpr int npieces(int n, int w) { return w == 32 ? n / 32 : (((n % 32) & w) ? 1 : 0); }
    __host__ __device__ static constexpr int piece_pos(int n, int w) {
        int p = (n / 32) * 32;
        if (w == 32) return 0;
        for (int x = 16; x > w; x >>= 1)
            if ((n % 32) & x) p += x;
        return p;
    }
    __host__ __device__ static constexpr int col0(int f, int w) {
        int c = 0;
        for (int x = 32; x > w; x >>= 1)
            for (int g = 0; g < kSNumFields; ++g) c += copies(g) * npieces(size(g), x) * x;
        for (int g = 0; g < f; ++g) c += copies(g) * npieces(size(g), w) * w;
        return c;
    }
    __host__ __device__ static constexpr int total() {
        int c = 0;
        for (int x = 32; x >= 1; x >>= 1)
            for (int g = 0; g < kSNumFields; ++g) c += copies(g) * npieces(size(g), x) * x;
        return c;
    }
    __host__ __device__ static constexpr int alloc() {
        int a = 32;
        while (a < total()) a *= 2;
        return a;
    }
    static_assert(total() <= 512, "history does not fit in tensor memory");
};

template <int D, int M, typename TIn>
struct SplitGeo {
    using Tl = Tile<D, M, false, true, TIn>;
    static_assert(D == M, "in-place gradient staging needs D == M");
    static constexpr int SF = replay_state_floats(D, M);
    // per group and stage: the token tile, then the gains (line box) and the
    // signed gain scales [chain][tau]
    static constexpr int oU = Tl::kBytes, oB = oU + kS * 32 * D * 4;
    static constexpr int kTileBytes = al1024(oB + 32 * kS * 4);
    static constexpr int kTx = Tl::kTx + kS * 32 * D * 4 + 32 * kS * 4;  // without gy, without state
    static constexpr int kSB = 32 * SF * 4;  // a group's start states [SF / 4][chain][4]
    static constexpr int kPerStage = 4 * kTileBytes;
    static constexpr int oT = 0;                        // [stage][group][tile]
    static constexpr int oSt = oT + 2 * kPerStage;      // [group][kSB]
    static constexpr int oBar = al128(oSt + 4 * kSB);   // [group][kBars]
    static constexpr int kBars = 5 + 2 * kXSlots;      // full[2] empty[2] sfree xfull[3] xempty[3]
    static constexpr int oSlot = oBar + 4 * kBars * 8;
    static constexpr int kSmem = oSlot + 16 + 1024;  // + alignment slack
    static constexpr bool kFits = kSmem <= kSmemMax;
};

// The covariance update of one token from its saved gain: P' = A P A + p I
// - beta u u^T (the arithmetic of cov_step).
template <int D>
__device__ __forceinline__ void cov_update(float (&P)[tri_size(D)], const float (&a)[D], float p,
                                           const float (&u)[D], float beta) {
    float nbu[D];
#pragma unroll
    for (int i = 0; i < D; ++i) nbu[i] = -beta * u[i];
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int j = i; j < D; ++j) {
            const int t = tri_index(D, i, j);
            const float upd = fmaf(nbu[i], u[j], (a[i] * a[j]) * P[t]);
            P[t] = (i == j) ? upd + p : upd;
        }
}

template <int D, int M, bool NEED_DYN, bool NEED_INIT, typename TIn>
__global__ void __launch_bounds__(kSplitThreads, 1)
    backward_split(const BwdArgs<TIn> A, const __grid_constant__ BwdMaps mp) {
    using G = SplitGeo<D, M, TIn>;
    using Tl = typename G::Tl;
    using TL = TLayoutSplit<D, M>;
    constexpr int TRI = tri_size(D), SF = G::SF, XF = 3 * D + 1;
    extern __shared__ __align__(128) char smem_raw[];
    char *const smem = smem_base(smem_raw);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int grp = warp & 3;
    const bool cov_warp = warp < 4;
    const int chain0 = static_cast<int>(blockIdx.x) * 128 + grp * 32;
    const long chain = chain0 + lane;
    const bool active = chain < A.n;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;
    const long rs_slots = replay_slots_per_chunk(T, L);
    const float floor_ = A.floor;
    const bool has_gy = A.gy != nullptr;
    char *const tiles = smem + G::oT + grp * G::kTileBytes;  // + stage * G::kPerStage
    float *const sbox = reinterpret_cast<float *>(smem + G::oSt + grp * G::kSB);  // [SF][32 chains]
    float *const state = sbox + 4 * lane;                                          // quads at +128 x
    uint64_t *const bars = reinterpret_cast<uint64_t *>(smem + G::oBar) + grp * G::kBars;
    uint64_t *const full = bars, *const empty = bars + 2, *const sfree = bars + 4;
    uint64_t *const xfull = bars + 5, *const xempty = bars + 5 + kXSlots;
    uint32_t *const slot = reinterpret_cast<uint32_t *>(smem + G::oSlot);
    const float *const bm = A.bmean + chain * (nb + 1) * D * M;
    const float *const bc = A.bcov + chain * (nb + 1) * D * D;

    if (cov_warp) {
        for (int x = 0; x < SF; ++x) state[rs_at(0, x)] = 0.f;  // idle lanes replay finite zeros
        if (lane == 0) {
            mbar_init(full, 1);
            mbar_init(full + 1, 1);
            mbar_init(empty, 2);
            mbar_init(empty + 1, 2);
            mbar_init(sfree, 2);
            for (int x = 0; x < kXSlots; ++x) {
                mbar_init(xfull + x, 32);
                mbar_init(xempty + x, 32);
            }
            mbar_init_fence();
        }
    }
    if (warp == 0) {
        tmem::alloc(slot, TL::alloc());
        tmem::relinquish();
    }
    tmem::fence_before_sync();
    __syncthreads();
    tmem::fence_after_sync();
    const uint32_t tb = *slot + (static_cast<uint32_t>(grp * 32) << 16);

    // An item's tile, gains (and saved start state) by the covariance warp's
    // lane 0; a checkpoint start state by each warp for its own part.
    auto issue_tile_state = [&](const BwdItems &it, int stage) {
        const bool saved = it.j > 0;
        char *const t = tiles + stage * G::kPerStage;
        const int t0 = static_cast<int>(it.t0());
        mbar_arrive_tx(full + stage, G::kTx + (has_gy ? Tl::szG : 0) + (saved ? G::kSB : 0));
        tma_load_2d(t + Tl::oK, &mp.k, t0 * D, chain0, full + stage);
        tma_load_2d(t + Tl::oQ, &mp.q, t0 * D, chain0, full + stage);
        tma_load_2d(t + Tl::oV, &mp.v, t0 * M, chain0, full + stage);
        tma_load_2d(t + Tl::oA, &mp.a, t0 * D, chain0, full + stage);
        tma_load_2d(t + Tl::oP, &mp.p, t0, chain0, full + stage);
        tma_load_2d(t + Tl::oR, &mp.r, t0, chain0, full + stage);
        if (has_gy) tma_load_2d(t + Tl::oG, &mp.gy, t0 * M, chain0, full + stage);
        tma_load_2d(t + G::oU, &mp.gu, t0 * D, chain0, full + stage);
        tma_load_2d(t + G::oB, &mp.gb, t0, chain0, full + stage);
        if (saved) tma_load_2d(sbox, &mp.rs, 0, state_row(chain0, nb, rs_slots, it.ci, it.j, SF), full + stage);
    };
    auto issue_checkpoint_part = [&](const BwdItems &it) {
        if (it.j > 0 || !active) return;
        const uint32_t s = smem_u32(state);  // float f at s + 4 rs_at(0, f)
        if (cov_warp) {
            const float *ck = bc + it.ci * D * D;
#pragma unroll
            for (int i = 0; i < D; ++i)
#pragma unroll
                for (int j = i; j < D; ++j) cp_async<4>(s + 4 * rs_at(0, D * M + tri_index(D, i, j)), ck + i * D + j);
        } else {
            const float *ck = bm + it.ci * D * M;
#pragma unroll
            for (int x = 0; x < D * M; ++x) cp_async<4>(s + 4 * rs_at(0, x), ck + x);
        }
    };
    // token tau's gain and scalars from the tile
    auto gains = [&](const char *t, int tau, float (&u)[D]) {
        line_load<D, float>(t + G::oU, lane, tau, u);
    };

    BwdItems cur, nxt;
    cur.init(T, L);
    nxt.init(T, L);
    if (!nxt.done) {
        if (cov_warp && lane == 0) issue_tile_state(nxt, 0);
        issue_checkpoint_part(nxt);
        cp_async_commit();
        nxt.advance();
    }
    long ntok = 0;  // exchange tokens so far (ring position)

    if (cov_warp) {
        // ------------------------------------------------------------------
        // covariance warp
        // ------------------------------------------------------------------
        float Rp[TRI];
#pragma unroll
        for (int t = 0; t < TRI; ++t) Rp[t] = 0.f;
        if (active && A.gcf != nullptr) {
            const float *gc = A.gcf + chain * D * D;
#pragma unroll
            for (int i = 0; i < D; ++i)
#pragma unroll
                for (int j = i; j < D; ++j) Rp[tri_index(D, i, j)] = 0.5f * (gc[i * D + j] + gc[j * D + i]);
        }
        long q = 0;
        while (!cur.done) {
            cp_async_wait<0>();
            mbar_wait(full + (q & 1), static_cast<uint32_t>((q >> 1) & 1));
            char *const tile = tiles + (q & 1) * G::kPerStage;
            const TileRead<D, M, false, true, TIn> rd{tile, lane};
            const int t0 = static_cast<int>(cur.t0());
            float4 p4, r4;
            rd.noise(p4, r4);
            const float4 b4 = reinterpret_cast<const float4 *>(tile + G::oB)[lane];
            float P[TRI];
            StateQuads<D, M>::get_cov(state, P);
            fence_proxy_async();  // these reads before the next state's TMA write (async proxy)
            __syncwarp();
            if (lane == 0) mbar_arrive(sfree);
            if (!nxt.done) issue_checkpoint_part(nxt);  // this warp's part of the row is read
            cp_async_commit();
            // next sub-chunk: once the mean warp has read its start state
            // and both warps released the stage the next tile goes to
            if (!nxt.done) {
                if (lane == 0) {
                    if (q >= 1) mbar_wait(empty + ((q + 1) & 1), static_cast<uint32_t>(((q - 1) >> 1) & 1));
                    mbar_wait(sfree, static_cast<uint32_t>(q & 1));
                    issue_tile_state(nxt, static_cast<int>((q + 1) & 1));
                }
                nxt.advance();
            }
            // replay: pre-step covariance per token, updated with the saved gains
#pragma unroll kUnrollReplay
            for (int tau = 0; tau < kS; ++tau) {
                float a[D], u[D];
                rd.decay(tau, a);
                gains(tile, tau, u);
                put<TL, kSPp, TRI>(tb, tau, P);
                cov_update<D>(P, a, sel4v(p4, tau), u, fabsf(sel4v(b4, tau)));
            }
            tmem::wait_st();
            // reverse: covariance adjoint
            float4 gp4 = make_float4(0.f, 0.f, 0.f, 0.f), gr4 = gp4;
#pragma unroll kUnrollCov
            for (int tau = kS - 1; tau >= 0; --tau, ++ntok) {
                const int xs = static_cast<int>(ntok % kXSlots);
                mbar_wait(xfull + xs, static_cast<uint32_t>((ntok / kXSlots) & 1));
                tmem::fence_after_sync();
                float xv[XF];
                get<TL, kSX, XF>(tb, xs, xv);
                tmem::fence_before_sync();
                mbar_arrive(xempty + xs);
                float k[D], a[D], u[D];
                rd.keys(tau, k);
                rd.decay(tau, a);
                gains(tile, tau, u);
                const float p = sel4v(p4, tau), bt = sel4v(b4, tau), beta = fabsf(bt);
                float Ru[D], trR = 0.f;
                float gb = xv[3 * D];
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    float acc = 0.f;
#pragma unroll
                    for (int j = 0; j < D; ++j) acc = fmaf(Rp[tri_index(D, i, j)], u[j], acc);
                    Ru[i] = acc;
                    gb = fmaf(-u[i], acc, gb);
                    if constexpr (NEED_DYN) trR += Rp[tri_index(D, i, i)];
                }
                const float gs = gain_scale_passes(bt) ? -beta * beta * gb : 0.f;
                float gu[D], ag[D];
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    gu[i] = beta * xv[i] - 2.f * beta * Ru[i] + gs * k[i];
                    ag[i] = a[i] * gu[i];
                }
                float Pp[TRI];
                get<TL, kSPp, TRI>(tb, tau, Pp);
                float gk[D];
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    float z = 0.f;
#pragma unroll
                    for (int j = 0; j < D; ++j) z = fmaf(Pp[tri_index(D, i, j)], ag[j], z);
                    const float gk3 = fmaf(a[i], z, p * gu[i]);
                    gk[i] = fmaf(-a[i], xv[D + i], fmaf(gs, u[i], gk3));
                }
                float gaP[D];
                float hg[D];  // gu / 2
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    gaP[i] = 0.f;
                    hg[i] = 0.5f * gu[i];
                }
#pragma unroll
                for (int i = 0; i < D; ++i)
#pragma unroll
                    for (int j = i; j < D; ++j) {
                        const int t = tri_index(D, i, j);
                        // S = R + sym(gu k^T), upper triangle
                        const float S =
                            i == j ? fmaf(gu[i], k[i], Rp[t]) : fmaf(hg[i], k[j], fmaf(hg[j], k[i], Rp[t]));
                        if constexpr (NEED_DYN) {
                            const float w = S * Pp[t];
                            gaP[i] = fmaf(w, a[j], gaP[i]);
                            if (i != j) gaP[j] = fmaf(w, a[i], gaP[j]);
                        }
                        Rp[t] = (a[i] * a[j]) * S;
                    }
                // keys and decay of this token are dead: their slots take gk, ga
                line_store<D, TIn>(tile + Tl::oK, lane, tau, gk);
                if constexpr (NEED_DYN) {
                    float ga[D], gpk = 0.f;
#pragma unroll
                    for (int i = 0; i < D; ++i) {
                        ga[i] = fmaf(2.f, gaP[i], xv[2 * D + i]);
                        gpk = fmaf(gu[i], k[i], gpk);
                    }
                    line_store<D, float>(tile + Tl::oA, lane, tau, ga);
                    const float gpv = trR + gpk;
                    gp4.x = tau == 0 ? gpv : gp4.x;
                    gp4.y = tau == 1 ? gpv : gp4.y;
                    gp4.z = tau == 2 ? gpv : gp4.z;
                    gp4.w = tau == 3 ? gpv : gp4.w;
                    gr4.x = tau == 0 ? gs : gr4.x;
                    gr4.y = tau == 1 ? gs : gr4.y;
                    gr4.z = tau == 2 ? gs : gr4.z;
                    gr4.w = tau == 3 ? gs : gr4.w;
                }
            }
            if constexpr (NEED_DYN) {
                reinterpret_cast<float4 *>(tile + Tl::oP)[lane] = gp4;
                reinterpret_cast<float4 *>(tile + Tl::oR)[lane] = gr4;
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                if (chain0 < A.n) {
                    tma_store_2d(&mp.gk, t0 * D, chain0, tile + Tl::oK);
                    if constexpr (NEED_DYN) {
                        tma_store_2d(&mp.ga, t0 * D, chain0, tile + Tl::oA);
                        tma_store_2d(&mp.gp, t0, chain0, tile + Tl::oP);
                        tma_store_2d(&mp.gr, t0, chain0, tile + Tl::oR);
                    }
                }
                bulk_commit();
                bulk_wait_read<0>();
                mbar_arrive(empty + (q & 1));
            }
            cur.advance();
            ++q;
        }
        cp_async_wait<0>();
        if constexpr (NEED_INIT) {
            if (active) store_cov_full<D>(A.gc0 + chain * D * D, Rp);
        }
    } else {
        // ------------------------------------------------------------------
        // mean warp
        // ------------------------------------------------------------------
        float gM[D][M];
#pragma unroll
        for (int i = 0; i < D; ++i)
#pragma unroll
            for (int c = 0; c < M; ++c) gM[i][c] = 0.f;
        if (active && A.gmf != nullptr) {
#pragma unroll
            for (int i = 0; i < D; ++i) load_vec<M>(A.gmf + chain * D * M + i * M, gM[i]);
        }
        long q = 0;
        while (!cur.done) {
            cp_async_wait<0>();
            mbar_wait(full + (q & 1), static_cast<uint32_t>((q >> 1) & 1));
            char *const tile = tiles + (q & 1) * G::kPerStage;
            const TileRead<D, M, false, true, TIn> rd{tile, lane};
            const int t0 = static_cast<int>(cur.t0());
            const float4 b4 = reinterpret_cast<const float4 *>(tile + G::oB)[lane];
            float Mm[D][M];
            StateQuads<D, M>::get_mean(state, Mm);
            fence_proxy_async();  // these reads before the next state's TMA write (async proxy)
            __syncwarp();
            if (lane == 0) mbar_arrive(sfree);
            if (!nxt.done) {
                issue_checkpoint_part(nxt);
                nxt.advance();
            }
            cp_async_commit();
            // replay: pre-step mean and innovation; gq = M' gy into the
            // token's (dead) value slot
#pragma unroll kUnrollReplay
            for (int tau = 0; tau < kS; ++tau) {
                float k[D], a[D], v[M], u[D], e[M];
                rd.keys(tau, k);
                rd.decay(tau, a);
                rd.values(tau, v);
                gains(tile, tau, u);
                const float beta = fabsf(sel4v(b4, tau));
                {
                    float flat[D * M];
#pragma unroll
                    for (int i = 0; i < D; ++i)
#pragma unroll
                        for (int c = 0; c < M; ++c) flat[i * M + c] = Mm[i][c];
                    put<TL, kSMp, D * M>(tb, tau, flat);
                }
                mean_step<D, M>(Mm, k, a, v, u, beta, e);
                put<TL, kSE, M>(tb, tau, e);
                float gq[D];
                if (has_gy) {
                    float gy[M];
                    rd.gy(tau, gy);
#pragma unroll
                    for (int i = 0; i < D; ++i) gq[i] = dot2<M>(Mm[i], gy);
                } else {
#pragma unroll
                    for (int i = 0; i < D; ++i) gq[i] = 0.f;
                }
                line_store<D, TIn>(tile + Tl::oV, lane, tau, gq);
            }
            tmem::wait_st();
            // reverse: mean adjoint; the covariance warp's inputs go through
            // the exchange ring
#pragma unroll kUnrollMean
            for (int tau = kS - 1; tau >= 0; --tau, ++ntok) {
                float k[D], a[D], u[D], e[M];
                rd.keys(tau, k);
                rd.decay(tau, a);
                gains(tile, tau, u);
                get<TL, kSE, M>(tb, tau, e);
                const float beta = fabsf(sel4v(b4, tau));
                if (has_gy) {
                    float qv[D], gy[M];
                    rd.queries(tau, qv);
                    rd.gy(tau, gy);
                    add_outer2<D, M>(gM, qv, gy);
                }
                float xv[XF];  // h, pk, gam, u.gM'.e
                float ge[M];
                const float gb = gain_adjoint2<D, M>(gM, u, e, beta, ge);
#pragma unroll
                for (int i = 0; i < D; ++i) xv[i] = dot2<M>(gM[i], e);
                constexpr int RB = 32 / M;  // rows per TMEM load
#pragma unroll
                for (int r0 = 0; r0 < D; r0 += RB) {
                    float Mp[RB][M];
                    if (r0 == 0) {
                        get_mean_rows<TL, kSMp, D, M, 0, RB>(tb, tau, Mp);
                    } else {
                        get_mean_rows<TL, kSMp, D, M, RB, RB>(tb, tau, Mp);
                    }
#pragma unroll
                    for (int ii = 0; ii < RB; ++ii) {
                        const int i = r0 + ii;
                        mean_row_adjoint2<M, NEED_DYN>(gM[i], Mp[ii], ge, k[i], a[i], xv[D + i], xv[2 * D + i]);
                    }
                }
                xv[3 * D] = gb;
                // the token's query slot is dead: it takes gv
                line_store<M, TIn>(tile + Tl::oQ, lane, tau, ge);
                const int xs = static_cast<int>(ntok % kXSlots);
                if (ntok >= kXSlots) {
                    mbar_wait(xempty + xs, static_cast<uint32_t>(((ntok - kXSlots) / kXSlots) & 1));
                    tmem::fence_after_sync();
                }
                put<TL, kSX, XF>(tb, xs, xv);
                tmem::wait_st();
                tmem::fence_before_sync();
                mbar_arrive(xfull + xs);
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) {
                if (chain0 < A.n) {
                    tma_store_2d(&mp.gq, t0 * D, chain0, tile + Tl::oV);
                    tma_store_2d(&mp.gv, t0 * M, chain0, tile + Tl::oQ);
                }
                bulk_commit();
                bulk_wait_read<0>();
                mbar_arrive(empty + (q & 1));
            }
            cur.advance();
            ++q;
        }
        cp_async_wait<0>();
        if constexpr (NEED_INIT) {
            if (active) store_mean<D, M>(A.gm0 + chain * D * M, gM);
        }
    }
    if (lane == 0) bulk_wait_all();
    tmem::fence_before_sync();
    __syncthreads();
    tmem::fence_after_sync();
    if (warp == 0) tmem::dealloc(*slot, TL::alloc());
}

// ===========================================================================
// Host side: tensor maps and launchers
// ===========================================================================
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeFn encode_fn() {
    static EncodeFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeFn>(nullptr);
        return reinterpret_cast<EncodeFn>(p);
    }();
    return fn;
}

template <typename T>
constexpr CUtensorMapDataType dtype_of() {
    return sizeof(T) == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
}

// Line map of a [N, T, rowelems] tensor: dims (row x token, chain), box
// (kS rows, 32 chains), swizzled with the line's span.
template <typename T>
bool map_tok(CUtensorMap *m, const T *base, int rowelems, long n, long t) {
    if (base == nullptr) return true;
    const cuuint64_t es = sizeof(T);
    const long span = static_cast<long>(kS) * rowelems * static_cast<long>(es);
    if (span != 16 && span != 32 && span != 64 && span != 128) return false;
    const CUtensorMapSwizzle sw = span == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : span == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                  : span == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                               : CU_TENSOR_MAP_SWIZZLE_NONE;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(rowelems) * t, static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(t) * rowelems * es};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(rowelems * kS), 32};
    const cuuint32_t estr[2] = {1, 1};
    return encode_fn()(m, dtype_of<T>(), 2, const_cast<T *>(base), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// Map of a [n, w] float tensor: dims (column, row), box (bw columns, bh rows).
inline bool map_rows(CUtensorMap *m, const float *base, long w, long n, int bw, int bh = 32) {
    if (base == nullptr) return true;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(w) * 4};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(bw), static_cast<cuuint32_t>(bh)};
    const cuuint32_t estr[2] = {1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Shapes the TMA path serves: rows of whole 4-byte words (lines of 16 bytes
// or more), every tile start on a 16-byte boundary of the noise rows,
// coordinates within int32.
template <typename TIn>
bool eligible(int d, int m, long n, long t, int chunks) {
    const int es = static_cast<int>(sizeof(TIn));
    return (d == 1 || d == 2 || d == 4 || d == 8) && m == 8 && (d * es) % 4 == 0 && (m * es) % 4 == 0 && t > 0 &&
           t % kS == 0 && chunks % kS == 0 && n < (1L << 30) && t < (1L << 30) && encode_fn() != nullptr;
}

template <int D, int M, bool FIXED, typename TIn>
int launch_fwd(const FwdArgs<TIn> &a, cudaStream_t st) {
    using G = FwdGeo<D, M, FIXED, TIn>;
    auto k = forward_chain<D, M, FIXED, TIn>;
    static bool attr = [&] {
        return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem) == cudaSuccess;
    }();
    if (!attr) return fail(BSSM_ERR_CUDA, "forward_chain: shared-memory attribute refused");
    if (a.out == nullptr) return fail(BSSM_ERR_INVALID, "forward_chain: null output");
    FwdMaps mp;
    std::memset(&mp, 0, sizeof(mp));
    const long nb = (a.t + a.chunks - 1) / a.chunks;
    bool ok = map_tok(&mp.k, a.keys, D, a.n, a.t) && map_tok(&mp.q, a.queries, D, a.n, a.t) &&
              map_tok(&mp.v, a.values, M, a.n, a.t) && map_tok(&mp.y, a.out, M, a.n, a.t);
    if (!FIXED)
        ok = ok && map_tok(&mp.a, a.decay, D, a.n, a.t) && map_rows(&mp.p, a.process, a.t, a.n, kS) &&
             map_rows(&mp.r, a.observation, a.t, a.n, kS);
    // The saved gains feed only the two-warp backward (backward_split: key dim
    // 8, learned dynamics, inputs its tiles fit); every other backward replays
    // from the saved states and forms the gains itself, so for those shapes
    // the forward skips the gain stores (12 bytes per chain-step at key dim 2).
    constexpr bool kGainsRead = D == 8 && !FIXED && SplitGeo<8, 8, TIn>::kFits;
    mp.gains = kGainsRead ? 1 : 0;
    if (a.rs != nullptr && kGainsRead) {
        ok = ok && map_tok(&mp.gu, static_cast<const float *>(replay_gains(a.rs, a.n, a.t, a.chunks, D, M)), D,
                           a.n, a.t) &&
             map_rows(&mp.gb, replay_gain_scales(a.rs, a.n, a.t, a.chunks, D, M), a.t, a.n, kS);
    }
    if (!ok) return fail(BSSM_ERR_CUDA, "forward_chain: tensor-map encoding failed");
    const long grid = (a.n + kThreads - 1) / kThreads;
    k<<<static_cast<unsigned>(grid), kThreads, G::kSmem, st>>>(a, mp);
    return check_launch("forward_chain");
}

// The backward allocates TMEM columns per CTA; co-resident CTAs on one SM
// must fit in the SM's 512 columns, or an allocation would wait for another
// CTA to finish.  Shared memory is raised until the occupancy guarantees it.
template <int D, int M, bool FIXED, bool NEED_DYN, bool NEED_INIT, typename TIn>
int launch_bwd(const BwdArgs<TIn> &a, cudaStream_t st) {
    using G = BwdGeo<D, M, FIXED, TIn>;
    using TL = TLayout<D, M>;
    auto k = backward_chain<D, M, FIXED, NEED_DYN, NEED_INIT, TIn>;
    static int smem = [&] {
        int bytes = G::kSmem;
        const int max_ctas = 512 / TL::alloc();
        for (;;) {
            if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return -1;
            int per_sm = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, bytes) != cudaSuccess) return -1;
            if (per_sm <= max_ctas) return per_sm >= 1 ? bytes : -1;
            bytes += 8 * 1024;
            if (bytes > kSmemMax) return -1;
        }
    }();
    if (smem < 0) return fail(BSSM_ERR_CUDA, "backward_chain: no launch configuration fits tensor memory");
    if (a.gk == nullptr || a.gv == nullptr || a.gq == nullptr ||
        (NEED_DYN && (a.ga == nullptr || a.gp == nullptr || a.gr == nullptr)) ||
        (NEED_INIT && (a.gm0 == nullptr || a.gc0 == nullptr)))
        return fail(BSSM_ERR_INVALID, "backward_chain: null gradient output");
    BwdMaps mp;
    std::memset(&mp, 0, sizeof(mp));
    const long nb = (a.t + a.chunks - 1) / a.chunks;
    const long W = replay_state_part(a.n, a.t, a.chunks, D, M) / 128;  // rows of 32 chains x 4
    bool ok = map_tok(&mp.k, a.keys, D, a.n, a.t) && map_tok(&mp.q, a.queries, D, a.n, a.t) &&
              map_tok(&mp.v, a.values, M, a.n, a.t) && map_tok(&mp.gy, a.gy, M, a.n, a.t);
    if (!FIXED)
        ok = ok && map_tok(&mp.a, a.decay, D, a.n, a.t) && map_rows(&mp.p, a.process, a.t, a.n, kS) &&
             map_rows(&mp.r, a.observation, a.t, a.n, kS);
    if (a.rs != nullptr && W > 0) ok = ok && map_rows(&mp.rs, a.rs, 128, W, 128, replay_state_floats(D, M) / 4);
    if (G::kStageOut) {
        ok = ok && map_tok(&mp.gk, a.gk, D, a.n, a.t) && map_tok(&mp.gv, a.gv, M, a.n, a.t) &&
             map_tok(&mp.gq, a.gq, D, a.n, a.t);
        if (NEED_DYN)
            ok = ok && map_tok(&mp.ga, a.ga, D, a.n, a.t) && map_rows(&mp.gp, a.gp, a.t, a.n, kS) &&
                 map_rows(&mp.gr, a.gr, a.t, a.n, kS);
    }
    if (!ok) return fail(BSSM_ERR_CUDA, "backward_chain: tensor-map encoding failed");
    const long grid = (a.n + kThreads - 1) / kThreads;
    k<<<static_cast<unsigned>(grid), kThreads, smem, st>>>(a, mp);
    return check_launch("backward_chain");
}

template <int D, int M, bool NEED_DYN, bool NEED_INIT, typename TIn>
int launch_split(const BwdArgs<TIn> &a, cudaStream_t st) {
    using G = SplitGeo<D, M, TIn>;
    auto k = backward_split<D, M, NEED_DYN, NEED_INIT, TIn>;
    static int smem = [&] {
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem) != cudaSuccess) return -1;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kSplitThreads, G::kSmem) != cudaSuccess)
            return -1;
        return per_sm == 1 ? G::kSmem : -1;  // one CTA per SM: it holds all 512 TMEM columns
    }();
    if (smem < 0) return fail(BSSM_ERR_CUDA, "backward_split: no launch configuration fits tensor memory");
    if (a.gk == nullptr || a.gv == nullptr || a.gq == nullptr ||
        (NEED_DYN && (a.ga == nullptr || a.gp == nullptr || a.gr == nullptr)) ||
        (NEED_INIT && (a.gm0 == nullptr || a.gc0 == nullptr)))
        return fail(BSSM_ERR_INVALID, "backward_split: null gradient output");
    BwdMaps mp;
    std::memset(&mp, 0, sizeof(mp));
    const long nb = (a.t + a.chunks - 1) / a.chunks;
    const long W = replay_state_part(a.n, a.t, a.chunks, D, M) / 128;  // rows of 32 chains x 4
    bool ok = map_tok(&mp.k, a.keys, D, a.n, a.t) && map_tok(&mp.q, a.queries, D, a.n, a.t) &&
              map_tok(&mp.v, a.values, M, a.n, a.t) && map_tok(&mp.gy, a.gy, M, a.n, a.t) &&
              map_tok(&mp.a, a.decay, D, a.n, a.t) && map_rows(&mp.p, a.process, a.t, a.n, kS) &&
              map_rows(&mp.r, a.observation, a.t, a.n, kS) && map_tok(&mp.gk, a.gk, D, a.n, a.t) &&
              map_tok(&mp.gv, a.gv, M, a.n, a.t) && map_tok(&mp.gq, a.gq, D, a.n, a.t);
    if (a.rs != nullptr && W > 0) ok = ok && map_rows(&mp.rs, a.rs, 128, W, 128, replay_state_floats(D, M) / 4);
    if (NEED_DYN)
        ok = ok && map_tok(&mp.ga, a.ga, D, a.n, a.t) && map_rows(&mp.gp, a.gp, a.t, a.n, kS) &&
             map_rows(&mp.gr, a.gr, a.t, a.n, kS);
    ok = ok && map_tok(&mp.gu, static_cast<const float *>(replay_gains(a.rs, a.n, a.t, a.chunks, D, M)), D, a.n,
                       a.t) &&
         map_rows(&mp.gb, replay_gain_scales(a.rs, a.n, a.t, a.chunks, D, M), a.t, a.n, kS);
    if (!ok) return fail(BSSM_ERR_CUDA, "backward_split: tensor-map encoding failed");
    const long grid = (a.n + 127) / 128;
    k<<<static_cast<unsigned>(grid), kSplitThreads, smem, st>>>(a, mp);
    return check_launch("backward_split");
}

// BSSM_KERNELS=chain1: the one-warp-per-group backward even where the split
// one applies (both are tested).
inline bool split_allowed() {
    const char *e = std::getenv("BSSM_KERNELS");
    return e == nullptr || std::strcmp(e, "chain1") != 0;
}

template <int D, int M, bool FIXED, typename TIn>
int launch_fwd_split(const FwdArgs<TIn> &a, cudaStream_t st) {
    using G = FSplitGeo<D, M, FIXED, TIn>;
    auto k = forward_split<D, M, FIXED, TIn>;
    static bool attr = [&] {
        return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmem) == cudaSuccess;
    }();
    if (!attr) return fail(BSSM_ERR_CUDA, "forward_split: shared-memory attribute refused");
    if (a.out == nullptr) return fail(BSSM_ERR_INVALID, "forward_split: null output");
    FwdMaps mp;
    std::memset(&mp, 0, sizeof(mp));
    bool ok = map_tok(&mp.k, a.keys, D, a.n, a.t) && map_tok(&mp.q, a.queries, D, a.n, a.t) &&
              map_tok(&mp.v, a.values, M, a.n, a.t) && map_tok(&mp.y, a.out, M, a.n, a.t);
    if (!FIXED)
        ok = ok && map_tok(&mp.a, a.decay, D, a.n, a.t) && map_rows(&mp.p, a.process, a.t, a.n, kS) &&
             map_rows(&mp.r, a.observation, a.t, a.n, kS);
    if (a.rs != nullptr) {
        ok = ok && map_tok(&mp.gu, static_cast<const float *>(replay_gains(a.rs, a.n, a.t, a.chunks, D, M)), D,
                           a.n, a.t) &&
             map_rows(&mp.gb, replay_gain_scales(a.rs, a.n, a.t, a.chunks, D, M), a.t, a.n, kS);
    }
    if (!ok) return fail(BSSM_ERR_CUDA, "forward_split: tensor-map encoding failed");
    const long grid = (a.n + 127) / 128;
    k<<<static_cast<unsigned>(grid), kSplitThreads, G::kSmem, st>>>(a, mp);
    return check_launch("forward_split");
}

template <int D, typename TIn>
constexpr bool fwd_fits() {
    if constexpr ((D * static_cast<int>(sizeof(TIn))) % 4 != 0) {
        return false;
    } else {
        return FwdGeo<D, 8, false, TIn>::kFits && FwdGeo<D, 8, true, TIn>::kFits;
    }
}

template <int D, typename TIn>
int fwd_d(int fixed, const FwdArgs<TIn> &a, cudaStream_t st) {
    if constexpr (!fwd_fits<D, TIn>()) {
        return fail(BSSM_ERR_UNSUPPORTED, "thread-per-chain forward: shape does not fit");
    } else {
        if constexpr (D == 8) {
            if constexpr (FSplitGeo<D, 8, false, TIn>::kFits && FSplitGeo<D, 8, true, TIn>::kFits) {
                if (split_allowed())
                    return fixed ? launch_fwd_split<D, 8, true, TIn>(a, st) : launch_fwd_split<D, 8, false, TIn>(a, st);
            }
        }
        return fixed ? launch_fwd<D, 8, true, TIn>(a, st) : launch_fwd<D, 8, false, TIn>(a, st);
    }
}

template <int D, bool FIXED, typename TIn>
int bwd_f(bool dyn, bool init, const BwdArgs<TIn> &a, cudaStream_t st) {
    if constexpr (D == 8 && !FIXED) {
        if constexpr (SplitGeo<D, 8, TIn>::kFits) {
            if (split_allowed() && a.rs != nullptr) {  // the replay buffer carries the gains
                if (dyn && init) return launch_split<D, 8, true, true, TIn>(a, st);
                if (dyn) return launch_split<D, 8, true, false, TIn>(a, st);
                if (init) return launch_split<D, 8, false, true, TIn>(a, st);
                return launch_split<D, 8, false, false, TIn>(a, st);
            }
        }
    }
    if (dyn && init) return launch_bwd<D, 8, FIXED, true, true, TIn>(a, st);
    if (dyn) return launch_bwd<D, 8, FIXED, true, false, TIn>(a, st);
    if (init) return launch_bwd<D, 8, FIXED, false, true, TIn>(a, st);
    return launch_bwd<D, 8, FIXED, false, false, TIn>(a, st);
}

template <int D, typename TIn>
int bwd_d(int fixed, bool dyn, bool init, const BwdArgs<TIn> &a, cudaStream_t st) {
    if constexpr ((D * static_cast<int>(sizeof(TIn))) % 4 != 0) {
        return fail(BSSM_ERR_UNSUPPORTED, "thread-per-chain kernels need key rows of whole words");
    } else {
        return fixed ? bwd_f<D, true, TIn>(dyn, init, a, st) : bwd_f<D, false, TIn>(dyn, init, a, st);
    }
}

}  // namespace chain

template <typename TIn>
bool chain_eligible(int d, long n, long t, int chunks, bool forward) {
    if (!chain::eligible<TIn>(d, 8, n, t, chunks)) return false;
    if (!forward) return true;
    switch (d) {
        case 1: return chain::fwd_fits<1, TIn>();
        case 2: return chain::fwd_fits<2, TIn>();
        case 4: return chain::fwd_fits<4, TIn>();
        case 8: return chain::fwd_fits<8, TIn>();
    }
    return false;
}

template <typename TIn>
int chain_forward(int d, int fixed, const FwdArgs<TIn> &a, cudaStream_t st) {
    if (a.n == 0) return BSSM_OK;
    if (!chain_eligible<TIn>(d, a.n, a.t, a.chunks, true))
        return fail(BSSM_ERR_UNSUPPORTED, "thread-per-chain kernels: shape not supported");
    switch (d) {
        case 1: return chain::fwd_d<1, TIn>(fixed, a, st);
        case 2: return chain::fwd_d<2, TIn>(fixed, a, st);
        case 4: return chain::fwd_d<4, TIn>(fixed, a, st);
        case 8: return chain::fwd_d<8, TIn>(fixed, a, st);
    }
    return fail(BSSM_ERR_UNSUPPORTED, "key_dim %d", d);
}

template <typename TIn>
int chain_backward(int d, int fixed, bool dyn, bool init, const BwdArgs<TIn> &a, cudaStream_t st) {
    if (a.n == 0 || (a.t == 0 && !init)) return BSSM_OK;
    if (!chain_eligible<TIn>(d, a.n, a.t, a.chunks, false))
        return fail(BSSM_ERR_UNSUPPORTED, "thread-per-chain kernels: shape not supported");
    if (a.rs == nullptr && replay_slots_per_chunk(a.t, a.chunks) > 0)
        return fail(BSSM_ERR_UNSUPPORTED, "thread-per-chain backward needs the forward's replay states");
    switch (d) {
        case 1: return chain::bwd_d<1, TIn>(fixed, dyn, init, a, st);
        case 2: return chain::bwd_d<2, TIn>(fixed, dyn, init, a, st);
        case 4: return chain::bwd_d<4, TIn>(fixed, dyn, init, a, st);
        case 8: return chain::bwd_d<8, TIn>(fixed, dyn, init, a, st);
    }
    return fail(BSSM_ERR_UNSUPPORTED, "key_dim %d", d);
}

}  // namespace bssm

extern "C" unsigned int bssm_debug_wait_timeouts(void) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, bssm::chain::g_wait_timeouts, sizeof(v)) != cudaSuccess) return ~0u;
    return v;
}

namespace {
// Give-ups already reported by bssm_stream_status, per device.
constexpr int kMaxDevices = 64;
std::mutex g_status_mu;
unsigned int g_status_seen[kMaxDevices] = {};
}  // namespace

extern "C" int bssm_stream_status(void *stream) {
    using bssm::fail;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return fail(BSSM_ERR_CUDA, "stream status: %s", cudaGetErrorString(err));
    if (dev < 0 || dev >= kMaxDevices) return fail(BSSM_ERR_INVALID, "stream status: device %d out of range", dev);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned int count = 0;
    // to pageable memory: returns once the stream's earlier work and the copy are done
    err = cudaMemcpyFromSymbolAsync(&count, bssm::chain::g_wait_timeouts, sizeof(count), 0, cudaMemcpyDeviceToHost,
                                    st);
    if (err == cudaSuccess) err = cudaStreamSynchronize(st);
    if (err != cudaSuccess) return fail(BSSM_ERR_CUDA, "stream status: %s", cudaGetErrorString(err));
    std::lock_guard<std::mutex> lock(g_status_mu);
    if (count != g_status_seen[dev]) {
        const unsigned int fresh = count - g_status_seen[dev];
        g_status_seen[dev] = count;
        return fail(BSSM_ERR_TIMEOUT,
                    "%u bounded wait(s) in a recurrence kernel gave up on device %d: the outputs of the calls "
                    "since the last status check are wrong",
                    fresh, dev);
    }
    bssm::g_last_error.clear();
    return BSSM_OK;
}

extern "C" int bssm_debug_wait_probe(int limit, void *stream) {
    using bssm::fail;
    if (limit < 1 || limit > (1 << 16)) return fail(BSSM_ERR_INVALID, "wait probe: limit %d not in [1, 65536]", limit);
    bssm::chain::wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit);
    return bssm::check_launch("wait probe");
}

namespace bssm {
template bool chain_eligible<float>(int, long, long, int, bool);
template bool chain_eligible<__nv_bfloat16>(int, long, long, int, bool);
template int chain_forward<float>(int, int, const FwdArgs<float> &, cudaStream_t);
template int chain_forward<__nv_bfloat16>(int, int, const FwdArgs<__nv_bfloat16> &, cudaStream_t);
template int chain_backward<float>(int, int, bool, bool, const BwdArgs<float> &, cudaStream_t);
template int chain_backward<__nv_bfloat16>(int, int, bool, bool, const BwdArgs<__nv_bfloat16> &, cudaStream_t);

}  // namespace bssm
