// bssm_envelope.cu -- the BayesianMixer's paper-feature prologue, fused.
//
// catid/bayes-ssm example/train_6layer.py:579-700 (fused Q/K/V + auxiliary
// projection, learned diagonal dynamics) turns one projection row per token
// into the recurrence's inputs with a chain of full-width PyTorch ops:
//   * a causal depthwise length-4 convolution over the Q/K/V channels
//     (CausalDepthwise4, :160-191: c[t] = sum_j w_j x[t + j - 3], zeros
//     before the sequence start);
//   * SiLU on each stream, then per-head L2 normalisation of q and k
//     (F.normalize, eps 1e-12);
//   * decay = exp(-softplus(logit + bias)), process / observation variance =
//     softplus(noise + bias) + 1e-4;
//   * the permute of every stream to chain-major [B*H, T, .].
// Here one kernel reads each projection row once and writes the recurrence's
// inputs in their final layout; one backward kernel recomputes the forward
// and writes the projection gradient plus per-tile partial sums for the
// convolution weight and auxiliary bias (reduced by a second, deterministic
// kernel).
//
// The readout epilogue (train_6layer.py:719-729) is the second kernel pair
// here: read [B*H, T, hd] -> read_norm (nn.RMSNorm over hd, after the
// reference's cast to the residual dtype) * SiLU(gate) -> [B, T, W].
//
// Work split: a thread owns adjacent channels of one batch row and walks
// a span of tokens, keeping the convolution window in registers, so every
// input element is read once (plus a 3-token halo per span).  The channels of
// one head sit in D/2 consecutive lanes, which reduce the head's squared norm
// with xor shuffles.  Streams and heads start at multiples of D/2 channel
// pairs, so a shuffle group never mixes a q/k head with other channels.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <type_traits>

#include "bayes_ssm_b200.h"
#include "bssm_flags.cuh"
#include "bssm_internal.h"

namespace bssm {
namespace env {

constexpr int kThreads = 256;
// Tokens per span (one thread walks one span) and the widest channel group,
// per direction, as measured at the config-3 mixer shape (B256 T512 H64 D8):
// forward 4 channels over 64 tokens (0.71 ms; 2 over 128: 0.87 ms; 8 over
// 32: 1.27 ms), backward 2 over 128 (before its load ring: 1.92 ms; 4 over
// 64: 2.0-3.4 ms; the walk unrolled by 2 or 4: 2.65 ms, with spills).
#ifndef BSSM_ENV_FWD_SPAN
#define BSSM_ENV_FWD_SPAN 64
#endif
#ifndef BSSM_ENV_BWD_SPAN
#define BSSM_ENV_BWD_SPAN 128
#endif
#ifndef BSSM_ENV_FWD_CW
#define BSSM_ENV_FWD_CW 4
#endif
// Tokens of loads each walk keeps in flight per thread (powers of two; per
// token and thread the forward's ring holds 16 bytes of shared memory, the
// backward's 2 x 8).  Where a token's elements fit in 8 bytes (BF16 inputs)
// the forward's ring holds twice BSSM_ENV_FWD_RING tokens in the same space
// (16 against 8: 0.412 against 0.419 ms at the config-3 mixer shape).
#ifndef BSSM_ENV_FWD_RING
#define BSSM_ENV_FWD_RING 8
#endif
#ifndef BSSM_ENV_BWD_RING
#define BSSM_ENV_BWD_RING 8
#endif
#ifndef BSSM_ENV_BWD_RING4  // the backward's ring with four channels per thread
#define BSSM_ENV_BWD_RING4 4
#endif
// Channels per thread in the backward where the shape allows four (2: always two).
#ifndef BSSM_ENV_BWD_CW
#define BSSM_ENV_BWD_CW 4
#endif
// Unroll factor of the backward's token walk: the tokens' recomputations are
// independent, so an unrolled walk overlaps them (4: 0.787 ms, 2: 0.809,
// 1: 0.824).
#ifndef BSSM_ENV_BWD_UNROLL
#define BSSM_ENV_BWD_UNROLL 4
#endif
// CTAs per SM the compiler sizes registers for (launch-bounds minimum; the
// backward's with two and with four channels per thread).  Before the load
// rings the walks were bound by load latency and occupancy won (5 / 4:
// forward 0.72 ms, backward 1.63 ms, against 0.89 / 2.61 ms at 1 / 1; issuing
// the backward's loads one token ahead in registers was neutral).  With the
// rings (8 tokens; 4 times the same) neither spills at 3 / 3 / 2: forward
// 0.44 ms (0.49 at 4), backward 0.97 ms with four channels per thread (1.35 at
// 3 CTAs, which spills) and 1.01 ms with two.
#ifndef BSSM_ENV_FWD_MINB
#define BSSM_ENV_FWD_MINB 3
#endif
#ifndef BSSM_ENV_BWD_MINB
#define BSSM_ENV_BWD_MINB 3
#endif
#ifndef BSSM_ENV_BWD_MINB4
#define BSSM_ENV_BWD_MINB4 2
#endif
constexpr int kFwdSpan = BSSM_ENV_FWD_SPAN, kBwdSpan = BSSM_ENV_BWD_SPAN;
constexpr int kFwdCW = BSSM_ENV_FWD_CW;
constexpr int kFwdRing = BSSM_ENV_FWD_RING, kRing = BSSM_ENV_BWD_RING, kRing4 = BSSM_ENV_BWD_RING4;
constexpr int kBwdCW = BSSM_ENV_BWD_CW, kBwdUnroll = BSSM_ENV_BWD_UNROLL;
static_assert(kRing4 >= 1 && (kRing4 & (kRing4 - 1)) == 0, "ring of a power of two tokens");
static_assert(kFwdRing >= 1 && (kFwdRing & (kFwdRing - 1)) == 0, "ring of a power of two tokens");
static_assert(kRing >= 1 && (kRing & (kRing - 1)) == 0, "ring of a power of two tokens");
constexpr int kRowGroups = 64;  // first-pass row groups of the gradient sums
constexpr float kNormEps = 1e-12f;  // F.normalize's default
constexpr float kNoiseFloor = 1e-4f;

enum Kind { kQ = 0, kK = 1, kV = 2, kDecay = 3, kNoise = 4, kIdle = 5 };

struct Shape {
    long b, t;
    int heads, d, hd;  // key dim D, value (head) dim
    long in_stride;    // elements between projection rows
    int tsplit;        // token spans per batch row
    __host__ __device__ int sw() const { return heads * d; }
    __host__ __device__ int width() const { return heads * hd; }
    __host__ __device__ int conv_channels() const { return 2 * sw() + width(); }
    __host__ __device__ int aux_channels() const { return sw() + 2 * heads; }
    __host__ __device__ int pairs() const { return (conv_channels() + aux_channels()) / 2; }
    // floats per row of the gradient partial sums: [C][4] weight taps, then
    // the auxiliary channels; padded to 8 so that every channel's taps are
    // 32-byte aligned
    __host__ __device__ int partial_cols() const { return (4 * conv_channels() + aux_channels() + 7) / 8 * 8; }
};

struct Chan {
    int kind, head, within;  // within: first of the pair's two channels inside its head row
};

__host__ __device__ __forceinline__ Chan classify(const Shape &s, int pair) {
    const int ch = 2 * pair, sw = s.sw(), w = s.width();
    if (ch < sw) return {kQ, ch / s.d, ch % s.d};
    if (ch < 2 * sw) return {kK, (ch - sw) / s.d, (ch - sw) % s.d};
    if (ch < 2 * sw + w) return {kV, (ch - 2 * sw) / s.hd, (ch - 2 * sw) % s.hd};
    const int a = ch - (2 * sw + w);
    if (a < sw) return {kDecay, a / s.d, a % s.d};
    if (a < sw + 2 * s.heads) return {kNoise, (a - sw) / 2, 0};
    return {kIdle, 0, 0};
}

// N consecutive elements (N = 2, 4 or 8) as floats; idx is a multiple of N
// and the base is aligned for the N-element vector.  Inputs are read-only for
// the whole launch, so they load through the non-coherent path: that also
// lets the compiler issue a later token's loads ahead of this token's stores,
// which it could not otherwise prove independent.
template <bool BF, int N>
__device__ __forceinline__ void ldn(const void *base, long idx, float *v) {
    if constexpr (BF) {
        const __nv_bfloat16 *p = static_cast<const __nv_bfloat16 *>(base) + idx;
        if constexpr (N == 2) {
            const unsigned raw = __ldg(reinterpret_cast<const unsigned *>(p));
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&raw));
            v[0] = f.x, v[1] = f.y;
        } else {
            using V = typename std::conditional<N == 4, uint2, uint4>::type;
            const V raw = __ldg(reinterpret_cast<const V *>(p));
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
            for (int i = 0; i < N / 2; ++i) {
                const float2 f = __bfloat1622float2(h[i]);
                v[2 * i] = f.x, v[2 * i + 1] = f.y;
            }
        }
    } else {
        const float *p = static_cast<const float *>(base) + idx;
        if constexpr (N == 2) {
            const float2 f = __ldg(reinterpret_cast<const float2 *>(p));
            v[0] = f.x, v[1] = f.y;
        } else {
#pragma unroll
            for (int i = 0; i < N; i += 4) {
                const float4 f = __ldg(reinterpret_cast<const float4 *>(p + i));
                v[i] = f.x, v[i + 1] = f.y, v[i + 2] = f.z, v[i + 3] = f.w;
            }
        }
    }
}
template <bool BF, int N>
__device__ __forceinline__ void stn(void *base, long idx, const float *v) {
    if constexpr (BF) {
        __nv_bfloat16 *p = static_cast<__nv_bfloat16 *>(base) + idx;
        if constexpr (N == 2) {
            *reinterpret_cast<__nv_bfloat162 *>(p) = __float22bfloat162_rn(make_float2(v[0], v[1]));
        } else {
            using V = typename std::conditional<N == 4, uint2, uint4>::type;
            V raw;
            __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&raw);
#pragma unroll
            for (int i = 0; i < N / 2; ++i) h[i] = __float22bfloat162_rn(make_float2(v[2 * i], v[2 * i + 1]));
            *reinterpret_cast<V *>(p) = raw;
        }
    } else {
        float *p = static_cast<float *>(base) + idx;
        if constexpr (N == 2) {
            *reinterpret_cast<float2 *>(p) = make_float2(v[0], v[1]);
        } else {
#pragma unroll
            for (int i = 0; i < N; i += 4) *reinterpret_cast<float4 *>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
    }
}
// CW / d whole heads of d channels (d = 2 or 4, d < CW) at consecutive
// chains: head gi of the thread is row ((chain + gi) * T + t) of width d.
// Every array offset is a compile-time constant, so v stays in registers.
template <bool BF, int CW>
__device__ __forceinline__ void st_heads(void *base, long chain, long t, long T, int d, const float *v) {
    if (d == 2) {
#pragma unroll
        for (int gi = 0; gi < CW / 2; ++gi) stn<BF, 2>(base, ((chain + gi) * T + t) * 2, v + 2 * gi);
    } else {
        if constexpr (CW >= 8) {
#pragma unroll
            for (int gi = 0; gi < CW / 4; ++gi) stn<BF, 4>(base, ((chain + gi) * T + t) * 4, v + 4 * gi);
        }
    }
}
template <bool BF, int CW>
__device__ __forceinline__ void ld_heads(const void *base, long chain, long t, long T, int d, float *v) {
    if (d == 2) {
#pragma unroll
        for (int gi = 0; gi < CW / 2; ++gi) ldn<BF, 2>(base, ((chain + gi) * T + t) * 2, v + 2 * gi);
    } else {
        if constexpr (CW >= 8) {
#pragma unroll
            for (int gi = 0; gi < CW / 4; ++gi) ldn<BF, 4>(base, ((chain + gi) * T + t) * 4, v + 4 * gi);
        }
    }
}

// The SiLU, normalisation and decay use the fast exponential and division
// intrinsics (a few ulp; the parity tests bound the result); the variances
// keep softplus exact, since a small variance is read relative to 1e-4.
__device__ __forceinline__ float sigmoid(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
// torch.nn.functional.softplus with beta 1, threshold 20
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float softplus_grad(float x) { return x > 20.f ? 1.f : 1.0f / (1.0f + expf(-x)); }
// exp(-softplus(z)) = 1 / (1 + e^z)
__device__ __forceinline__ float decay_of(float z) { return __fdividef(1.0f, 1.0f + __expf(z)); }
// 1 / max(sqrt(ss), eps) for F.normalize
__device__ __forceinline__ float inv_norm(float ss) { return rsqrtf(fmaxf(ss, kNormEps * kNormEps)); }

// Sum over `lanes` consecutive lanes (a power of two; all lanes call it).
__device__ __forceinline__ float lane_sum(float v, int lanes) {
    for (int off = 1; off < lanes; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}
// The same with the lane count fixed at compile time (L > 0) or read at run
// time (L = 0).
template <int L>
__device__ __forceinline__ float lane_sum_n(float v, int lanes) {
    if constexpr (L == 0) {
        return lane_sum(v, lanes);
    } else {
#pragma unroll
        for (int off = 1; off < L; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        return v;
    }
}

// How a thread's CW channels map onto heads of D (q, k, decay): one head
// spread over D / CW lanes (D >= CW), or CW / D whole heads (D < CW).
struct HeadMap {
    int dg;     // channels per head group inside the thread
    int ng;     // head groups inside the thread
    int lanes;  // lanes per head
    int shift;  // log2(dg): channel j of the thread is in head group j >> shift
};
template <int CW>
__device__ __forceinline__ HeadMap head_map(int d) {
    return d >= CW ? HeadMap{CW, 1, d / CW, 31 - __clz(CW)} : HeadMap{d, CW / d, 1, 31 - __clz(d)};
}

// Work of one warp: 32 consecutive channel groups of one (batch row, token
// span).  Warps, not CTAs, tile the (row, span) pairs, so a pair whose groups
// are not a multiple of the CTA's 256 leaves no partly-empty CTA behind.
struct Work {
    long bb;
    int span, grp;
    bool live;
};
template <int CW>
__device__ __forceinline__ Work work_of(const Shape &s) {
    const int wpr = ((s.conv_channels() + s.aux_channels()) / CW + 31) / 32;  // warps per (row, span)
    const long gw = static_cast<long>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
    const long row = gw / wpr;
    const int wi = static_cast<int>(gw - row * wpr);
    return {row / s.tsplit, static_cast<int>(row % s.tsplit), wi * 32 + static_cast<int>(threadIdx.x & 31),
            row < s.b * s.tsplit};
}

// Per-thread load rings.  Both walks stream their per-token loads a few
// tokens ahead through shared memory (cp.async, zero-filled where a token or
// a gradient is absent), so each warp keeps several tokens of loads in
// flight instead of one.  Each thread reads back only its own copies, so a
// ring needs no barrier: cp.async.wait_group orders them.
__device__ __forceinline__ uint32_t shared_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
template <int G>
__device__ __forceinline__ void cp_async_zfill(uint32_t dst, const void *src, bool on) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;\n" ::"r"(dst), "l"(src), "n"(G), "r"(on ? G : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// N elements (BF16 or FP32) from the front of a ring slot, as floats.
template <bool BF, int N, class W>
__device__ __forceinline__ void unpack(const W &raw, float *v) {
    const unsigned *u = reinterpret_cast<const unsigned *>(&raw);
    static_assert(sizeof(W) >= N * (BF ? 2 : 4), "slot too small");
#pragma unroll
    for (int i = 0; i < (BF ? N / 2 : N); ++i) {
        if constexpr (BF) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(u + i));
            v[2 * i] = f.x, v[2 * i + 1] = f.y;
        } else {
            v[i] = __uint_as_float(u[i]);
        }
    }
}

struct ProArgs {
    const void *x;
    const float *w;     // [C][4]
    const float *bias;  // [SW + 2H] or null
    void *k, *q, *v;    // [B*H, T, D] / [B*H, T, HD]
    float *decay;       // [B*H, T, D]
    float *process, *observation;  // [B*H, T]
    // null, or the check words of keys, values, queries, decay, process and
    // observation (in that order): the CHECK_* flags of the values written
    unsigned *flags;
};

// The input checks of bayesian_layer over the values this kernel writes, as
// bssm_check_values reports them.  The projection streams and the decay are
// checked for finiteness only, through an accumulator that fma(v, 0, acc)
// turns NaN exactly when some v is infinite or NaN (0 * finite is a zero and
// never overflows); the noise rows get all three flags (check_flags_of).
template <bool OUT_BF, int N>
__device__ __forceinline__ void nonfinite_acc(float &acc, const float (&v)[N]) {
#pragma unroll
    for (int j = 0; j < N; ++j) {
        // the value as stored: a BF16 output can round a finite value to infinity
        const float x = OUT_BF ? __bfloat162float(__float2bfloat16_rn(v[j])) : v[j];
        acc = fmaf(x, 0.f, acc);
    }
}

// Thread = CW adjacent channels of one stream (every stream and head row
// boundary falls on a multiple of CW), walking one token span.
// L > 0: every q / k head spans exactly L lanes (key dim L * CW), fixed at
// compile time; L = 0: read from the shape, heads of fewer than CW channels
// included.
template <bool IN_BF, bool OUT_BF, int CW, int L>
__global__ void __launch_bounds__(kThreads, BSSM_ENV_FWD_MINB) prologue_kernel(const Shape s, const ProArgs a) {
    const Work wk = work_of<CW>(s);
    if (!wk.live) return;  // past the last (batch row, span): the whole warp (no block barriers here)
    const int grp = wk.grp;
    const long bb = wk.bb;
    const long span = (s.t + s.tsplit - 1) / s.tsplit;
    const long t0 = wk.span * span;
    const long t1 = t0 + span < s.t ? t0 + span : s.t;
    const int c0 = CW * grp;
    const Chan ch = c0 < s.conv_channels() + s.aux_channels() ? classify(s, c0 / 2) : Chan{kIdle, 0, 0};
    const HeadMap hm = head_map<CW>(s.d);
    // does any lane of this warp hold q / k channels (the head norms run only then)
    const bool warp_qk = __any_sync(0xffffffffu, ch.kind == kQ || ch.kind == kK);
    const long row0 = bb * s.t;
    const long chain = bb * s.heads + ch.head;
    const bool conv = ch.kind <= kV;
    float w[4][CW], bias[CW];
#pragma unroll
    for (int j = 0; j < CW; ++j) {
        bias[j] = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k][j] = 0.f;
    }
    if (conv) {
#pragma unroll
        for (int j = 0; j < CW; ++j) {
            const float4 wj = *reinterpret_cast<const float4 *>(a.w + (c0 + j) * 4);
            w[0][j] = wj.x, w[1][j] = wj.y, w[2][j] = wj.z, w[3][j] = wj.w;
        }
    } else if (ch.kind != kIdle && a.bias != nullptr) {
#pragma unroll
        for (int j = 0; j < CW; ++j) bias[j] = a.bias[c0 - s.conv_channels() + j];
    }
    float xm3[CW], xm2[CW], xm1[CW], x[CW], o[CW];
#pragma unroll
    for (int j = 0; j < CW; ++j) xm3[j] = xm2[j] = xm1[j] = 0.f;
    if (conv) {
        if (t0 - 3 >= 0) ldn<IN_BF, CW>(a.x, (row0 + t0 - 3) * s.in_stride + c0, xm3);
        if (t0 - 2 >= 0) ldn<IN_BF, CW>(a.x, (row0 + t0 - 2) * s.in_stride + c0, xm2);
        if (t0 - 1 >= 0) ldn<IN_BF, CW>(a.x, (row0 + t0 - 1) * s.in_stride + c0, xm1);
    }
    // ring of the next FR tokens' projection elements (step k = token t0 + k)
    constexpr int XS = CW * (IN_BF ? 2 : 4);
    static_assert(XS <= 16, "one cp.async per token");
    // 8-byte slots hold twice the tokens in the same shared memory
    using FSlot = typename std::conditional<(XS <= 8), uint2, uint4>::type;
    constexpr int FR = XS <= 8 ? 2 * kFwdRing : kFwdRing;
    __shared__ FSlot ring[FR][kThreads];
    const char *const xb = static_cast<const char *>(a.x);
    const long xstep = s.in_stride * (XS / CW);
    const char *const xrow = xb + row0 * xstep + c0 * static_cast<long>(XS / CW);
    const int steps = static_cast<int>(t1 - t0);
    const char *xp = xrow + t0 * xstep;  // the next token to issue
    auto issue = [&](int k) {
        const bool on = k < steps && ch.kind != kIdle;
        cp_async_zfill<XS>(shared_addr(&ring[k & (FR - 1)][threadIdx.x]), on ? xp : xb, on);
        xp += xstep;
        cp_async_commit_group();
    };
#pragma unroll
    for (int k = 0; k < FR; ++k) issue(k);
    // element index of this thread's output row at the current token (q / k /
    // decay rows of d, v rows of hd), and of its chains' variances
    const long ostep = ch.kind == kV ? s.hd : s.d;
    long oidx = (chain * s.t + t0) * ostep + ch.within;
    long nidx = chain * s.t + t0;
    float nfacc = 0.f;               // NaN once a written q / k / v / decay value is not finite
    unsigned pflags = 0, rflags = 0;  // of the process and observation values written
#pragma unroll 4
    for (int k = 0; k < steps; ++k, oidx += ostep, ++nidx) {
        const long t = t0 + k;
        cp_async_wait_group<FR - 1>();
        unpack<IN_BF, CW>(ring[k & (FR - 1)][threadIdx.x], x);
        float ss[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) {
            const float c = fmaf(w[3][j], x[j], fmaf(w[2][j], xm1[j], fmaf(w[1][j], xm2[j], w[0][j] * xm3[j])));
            o[j] = c * sigmoid(c);
            ss[j] = o[j] * o[j];
            xm3[j] = xm2[j];
            xm2[j] = xm1[j];
            xm1[j] = x[j];
        }
        const bool qk = ch.kind == kQ || ch.kind == kK;
        if ((L > 0 || hm.ng == 1) && warp_qk) {  // one head (part) per thread: reduce across its lanes
            float tot = 0.f;
#pragma unroll
            for (int j = 0; j < CW; ++j) tot += ss[j];
            tot = lane_sum_n<L>(qk ? tot : 0.f, hm.lanes);
            if (qk) {
                const float r = inv_norm(tot);
#pragma unroll
                for (int j = 0; j < CW; ++j) o[j] *= r;
                stn<OUT_BF, CW>(ch.kind == kQ ? a.q : a.k, oidx, o);
                nonfinite_acc<OUT_BF>(nfacc, o);
            }
        } else if (L == 0 && hm.ng > 1 && qk) {  // CW / D whole heads
#pragma unroll
            for (int gi = 0; gi < CW / 2; ++gi) {
                if (gi >= hm.ng) break;
                float tot = 0.f;
#pragma unroll
                for (int j = 0; j < CW; ++j)
                    if ((j >> hm.shift) == gi) tot += ss[j];
                const float r = inv_norm(tot);
#pragma unroll
                for (int j = 0; j < CW; ++j)
                    if ((j >> hm.shift) == gi) o[j] *= r;
            }
            st_heads<OUT_BF, CW>(ch.kind == kQ ? a.q : a.k, chain, t, s.t, s.d, o);
            nonfinite_acc<OUT_BF>(nfacc, o);
        }
        if (ch.kind == kV) {
            stn<OUT_BF, CW>(a.v, oidx, o);
            nonfinite_acc<OUT_BF>(nfacc, o);
        } else if (ch.kind == kDecay) {
            float dcy[CW];
#pragma unroll
            for (int j = 0; j < CW; ++j) dcy[j] = decay_of(x[j] + bias[j]);
            if (L > 0 || hm.ng == 1) {
                stn<false, CW>(a.decay, oidx, dcy);
            } else {
                st_heads<false, CW>(a.decay, chain, t, s.t, s.d, dcy);
            }
            nonfinite_acc<false>(nfacc, dcy);
        } else if (ch.kind == kNoise) {
#pragma unroll
            for (int i = 0; i < CW / 2; ++i) {
                const float pv = softplus(x[2 * i] + bias[2 * i]) + kNoiseFloor;
                const float rv = softplus(x[2 * i + 1] + bias[2 * i + 1]) + kNoiseFloor;
                a.process[nidx + i * s.t] = pv;
                a.observation[nidx + i * s.t] = rv;
                pflags |= check_flags_of(pv);
                rflags |= check_flags_of(rv);
            }
        }
        issue(k + FR);  // after the slot's values were used
    }
    cp_async_wait_group<0>();
    if (a.flags != nullptr) {  // flags are rare: one atomic per thread that saw one
        if (ch.kind == kNoise) {
            if (pflags) atomicOr(a.flags + 4, pflags);
            if (rflags) atomicOr(a.flags + 5, rflags);
        } else if (ch.kind != kIdle && nfacc != nfacc) {
            const int slot = ch.kind == kK ? 0 : ch.kind == kV ? 1 : ch.kind == kQ ? 2 : 3;
            atomicOr(a.flags + slot, BSSM_CHECK_NONFINITE);
        }
    }
}

struct EnvBwdArgs {
    const void *x;
    const float *w, *bias;
    const void *gk, *gq, *gv;  // null = zero
    const float *gdecay, *gprocess, *gobservation;
    void *gx;        // [B, T, gx_stride] (the prologue's channels only)
    long gx_stride;
    float *partial;  // [B * tsplit][partial_cols]
};

// Backward of one token span: walk the tokens downwards, recompute the
// forward at each, and keep the last four convolution-input gradients so that
// gx[t] = sum_j w_j gc[t + 3 - j].  The span also recomputes the 3 tokens
// after it (their gc feeds its last gx) without counting them in the weight
// gradient, which their own span does.
//
// A thread owns CW = 2 or 4 adjacent channels, never more than one q / k head
// (the host takes CW = 4 only for key dims >= 4), so a head spans d / CW
// whole lanes; L is that lane count when the host fixes it at compile time
// (0: read from the shape).  Its ring holds, per token, the projection
// elements and the incoming gradients of its channels.
template <bool IN_BF, bool OUT_BF, int CW, int L>
__global__ void __launch_bounds__(kThreads, CW == 4 ? BSSM_ENV_BWD_MINB4 : BSSM_ENV_BWD_MINB)
    prologue_backward_kernel(const Shape s, const EnvBwdArgs a) {
    static_assert(CW == 2 || CW == 4, "two or four channels per thread");
    constexpr int XS = CW * (IN_BF ? 2 : 4), GS = CW * (OUT_BF ? 2 : 4);  // bytes per token
    constexpr int R = CW == 2 ? kRing : kRing4;
    using Slot = typename std::conditional<CW == 2, uint2, uint4>::type;
    __shared__ Slot ring_x[R][kThreads], ring_g[R][kThreads];
    const Work wk = work_of<CW>(s);
    if (!wk.live) return;  // past the last (batch row, span): the whole warp (no block barriers here)
    const int grp = wk.grp;
    const long bb = wk.bb;
    const long span = (s.t + s.tsplit - 1) / s.tsplit;
    const long t0 = wk.span * span;
    const long t1 = t0 + span < s.t ? t0 + span : s.t;
    const long hi = t1 + 3 < s.t ? t1 + 3 : s.t;
    const int c0 = CW * grp;
    const int C = s.conv_channels();
    const Chan ch = c0 < C + s.aux_channels() ? classify(s, c0 / 2) : Chan{kIdle, 0, 0};
    const int lanes = L > 0 ? L : s.d / CW;  // lanes per q / k head
    // does any lane of this warp hold q / k channels (the head norms run only then)
    const bool warp_qk = __any_sync(0xffffffffu, ch.kind == kQ || ch.kind == kK);
    const long row0 = bb * s.t;
    const long chain = bb * s.heads + ch.head;
    const bool conv = ch.kind <= kV;
    const bool qk = ch.kind == kQ || ch.kind == kK;
    const bool aux = ch.kind == kDecay || ch.kind == kNoise;
    float *const part = a.partial + (bb * s.tsplit + wk.span) * static_cast<long>(s.partial_cols());
    float w[4][CW], bias[CW], gw[4][CW], gb[CW];
#pragma unroll
    for (int j = 0; j < CW; ++j) {
        bias[j] = gb[j] = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k][j] = gw[k][j] = 0.f;
    }
    if (conv) {
#pragma unroll
        for (int j = 0; j < CW; ++j) {
            const float4 wj = *reinterpret_cast<const float4 *>(a.w + (c0 + j) * 4);
            w[0][j] = wj.x, w[1][j] = wj.y, w[2][j] = wj.z, w[3][j] = wj.w;
        }
    } else if (aux && a.bias != nullptr) {
#pragma unroll
        for (int j = 0; j < CW; ++j) bias[j] = a.bias[c0 - C + j];
    }
    // Byte addresses of these channels at token 0 and per token: the
    // projection row, and the incoming gradient -- a [B*H, T, .] row for
    // q / k / v or the decay, or the per-chain variances (gsrc: the process
    // variance of the first chain, gsrc2: its observation variance; the
    // second chain's, for CW = 4, sit T floats further on).
    const char *const xb = static_cast<const char *>(a.x);
    const long xstep = s.in_stride * (XS / CW);
    const char *const xrow = xb + row0 * xstep + c0 * static_cast<long>(XS / CW);
    const char *gsrc = nullptr, *gsrc2 = nullptr;
    long gstep = 0;
    if (conv) {
        gstep = (ch.kind == kV ? s.hd : s.d) * static_cast<long>(GS / CW);
        gsrc = static_cast<const char *>(ch.kind == kQ ? a.gq : ch.kind == kK ? a.gk : a.gv);
        if (gsrc) gsrc += chain * s.t * gstep + ch.within * static_cast<long>(GS / CW);
    } else if (ch.kind == kDecay) {
        gstep = s.d * 4L;
        gsrc = reinterpret_cast<const char *>(a.gdecay);
        if (gsrc) gsrc += chain * s.t * gstep + ch.within * 4L;
    } else if (ch.kind == kNoise) {
        gstep = 4;
        gsrc = reinterpret_cast<const char *>(a.gprocess);
        gsrc2 = reinterpret_cast<const char *>(a.gobservation);
        if (gsrc) gsrc += chain * s.t * 4L;
        if (gsrc2) gsrc2 += chain * s.t * 4L;
    }
    const long chain_bytes = s.t * 4L;  // between two chains' variance rows
    // Step k of the walk is token hi - 1 - k: conv channels need x[t - 3]
    // (x[t .. t - 2] are in registers), the auxiliary ones x[t] inside the span.
    const int steps = static_cast<int>(hi - t0);
    const char *xp = xrow + (conv ? hi - 4 : hi - 1) * xstep;  // step 0's loads; each step moves one token down
    const char *gq1 = gsrc ? gsrc + (hi - 1) * gstep : nullptr;
    const char *gq2 = gsrc2 ? gsrc2 + (hi - 1) * gstep : nullptr;
    auto issue = [&](int k) {
        const long t = hi - 1 - k;
        const int slot = k & (R - 1);
        const bool live = k < steps && ch.kind != kIdle;
        const bool xon = live && (conv ? t >= 3 : t < t1);
        cp_async_zfill<XS>(shared_addr(&ring_x[slot][threadIdx.x]), xon ? xp : xb, xon);
        const bool gon = live && (conv || t < t1);
        const bool on1 = gon && gq1 != nullptr, on2 = gon && gq2 != nullptr;
        const uint32_t gdst = shared_addr(&ring_g[slot][threadIdx.x]);
        if (ch.kind == kNoise) {  // (process, observation) of CW / 2 chains
#pragma unroll
            for (int i = 0; i < CW / 2; ++i) {
                cp_async_zfill<4>(gdst + 8 * i, on1 ? gq1 + i * chain_bytes : xb, on1);
                cp_async_zfill<4>(gdst + 8 * i + 4, on2 ? gq2 + i * chain_bytes : xb, on2);
            }
        } else if (ch.kind == kDecay) {
            cp_async_zfill<4 * CW>(gdst, on1 ? gq1 : xb, on1);
        } else {
            cp_async_zfill<GS>(gdst, on1 ? gq1 : xb, on1);
        }
        xp -= xstep;
        if (gq1) gq1 -= gstep;
        if (gq2) gq2 -= gstep;
        cp_async_commit_group();
    };
    // x0 = x[t], x1 = x[t-1], x2 = x[t-2], x3 = x[t-3] (conv channels)
    float x0[CW], x1[CW], x2[CW], x3[CW];
    float gp1[CW], gp2[CW], gp3[CW];  // gc[t+1], gc[t+2], gc[t+3]
#pragma unroll
    for (int j = 0; j < CW; ++j) x0[j] = x1[j] = x2[j] = x3[j] = gp1[j] = gp2[j] = gp3[j] = 0.f;
    auto ldx = [&](long t, float *v) {
        if (t >= 0) ldn<IN_BF, CW>(a.x, (row0 + t) * s.in_stride + c0, v);
    };
    if (conv && hi > t0) {
        ldx(hi - 1, x0);
        ldx(hi - 2, x1);
        ldx(hi - 3, x2);
    }
#pragma unroll
    for (int k = 0; k < R; ++k) issue(k);
    long gxi = (row0 + hi - 1) * a.gx_stride + c0;  // element of gx at the current token
#pragma unroll(kBwdUnroll)
    for (int k = 0; k < steps; ++k, gxi -= a.gx_stride) {
        const long t = hi - 1 - k;
        cp_async_wait_group<R - 1>();
        const int slot = k & (R - 1);
        const Slot rx = ring_x[slot][threadIdx.x], rg = ring_g[slot][threadIdx.x];
        float gc[CW], g[CW], o[CW], ds[CW];
#pragma unroll
        for (int j = 0; j < CW; ++j) gc[j] = o[j] = ds[j] = 0.f;
        unpack<false, CW>(rg, g);  // decay / variance gradients (FP32)
        if (conv) {
            unpack<IN_BF, CW>(rx, x3);
            unpack<OUT_BF, CW>(rg, g);
#pragma unroll
            for (int j = 0; j < CW; ++j) {
                const float c = fmaf(w[3][j], x0[j], fmaf(w[2][j], x1[j], fmaf(w[1][j], x2[j], w[0][j] * x3[j])));
                const float sg = sigmoid(c);
                o[j] = c * sg;
                ds[j] = sg * fmaf(c, 1.f - sg, 1.f);  // silu'
            }
        }
        // q, k: y = s / max(|s|, eps); dy/ds = (I - y y^T) / |s| above eps, I / eps below
        if (warp_qk) {
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < CW; ++j) ss += o[j] * o[j];
            ss = lane_sum_n<L>(qk ? ss : 0.f, lanes);
            const float r = inv_norm(ss);
            const bool above = ss > kNormEps * kNormEps;
            float dot = 0.f;
#pragma unroll
            for (int j = 0; j < CW; ++j) dot += o[j] * r * g[j];
            dot = lane_sum_n<L>(qk ? dot : 0.f, lanes);
            if (qk) {
                const float dd = above ? dot : 0.f;
#pragma unroll
                for (int j = 0; j < CW; ++j) gc[j] = (g[j] - o[j] * r * dd) * r * ds[j];
            }
        }
        if (ch.kind == kV) {
#pragma unroll
            for (int j = 0; j < CW; ++j) gc[j] = g[j] * ds[j];
        }
        if (t < t1) {
            if (conv) {
                float gx[CW];
#pragma unroll
                for (int j = 0; j < CW; ++j) {
                    gx[j] = fmaf(w[0][j], gp3[j], fmaf(w[1][j], gp2[j], fmaf(w[2][j], gp1[j], w[3][j] * gc[j])));
                    gw[0][j] = fmaf(gc[j], x3[j], gw[0][j]);
                    gw[1][j] = fmaf(gc[j], x2[j], gw[1][j]);
                    gw[2][j] = fmaf(gc[j], x1[j], gw[2][j]);
                    gw[3][j] = fmaf(gc[j], x0[j], gw[3][j]);
                }
                stn<IN_BF, CW>(a.gx, gxi, gx);
            } else if (aux) {
                float xv[CW], gz[CW];
                unpack<IN_BF, CW>(rx, xv);
                if (ch.kind == kDecay) {
#pragma unroll
                    for (int j = 0; j < CW; ++j) {
                        // d/dz 1 / (1 + e^z) = -decay (1 - decay)
                        const float dcy = decay_of(xv[j] + bias[j]);
                        gz[j] = -g[j] * dcy * (1.f - dcy);
                    }
                } else {  // (process, observation) pairs
#pragma unroll
                    for (int j = 0; j < CW; ++j) gz[j] = g[j] * softplus_grad(xv[j] + bias[j]);
                }
#pragma unroll
                for (int j = 0; j < CW; ++j) gb[j] += gz[j];
                stn<IN_BF, CW>(a.gx, gxi, gz);
            }
        }
#pragma unroll
        for (int j = 0; j < CW; ++j) {
            gp3[j] = gp2[j];
            gp2[j] = gp1[j];
            gp1[j] = gc[j];
            x0[j] = x1[j];
            x1[j] = x2[j];
            x2[j] = x3[j];
        }
        issue(k + R);  // after the slot's values were used
    }
    cp_async_wait_group<0>();
    if (conv) {
#pragma unroll
        for (int j = 0; j < CW; ++j)  // [c][4]: 16-byte aligned (rows are multiples of 8 floats)
            *reinterpret_cast<float4 *>(part + (c0 + j) * 4) = make_float4(gw[0][j], gw[1][j], gw[2][j], gw[3][j]);
    } else if (aux) {
#pragma unroll
        for (int j = 0; j < CW; ++j) part[4 * C + (c0 - C) + j] = gb[j];
    }
}

// ---- readout epilogue -----------------------------------------------------
template <bool BF, int N>
__device__ __forceinline__ void ldv(const void *base, long idx, float *v) {
    static_assert(N % 8 == 0, "rows of 8k");
#pragma unroll
    for (int i = 0; i < N; i += 8) ldn<BF, 8>(base, idx + i, v + i);
}
template <bool BF, int N>
__device__ __forceinline__ void stv(void *base, long idx, const float *v) {
#pragma unroll
    for (int i = 0; i < N; i += 8) stn<BF, 8>(base, idx + i, v + i);
}
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

struct EpiArgs {
    const void *read;  // [B*H, T, HD]
    const void *gate;  // rows of [B, T, >= W], gate_stride apart
    long gate_stride;
    const float *w;    // [HD]
    float eps;
    long b, t;
    int heads;
    void *out;         // [B, T, W] (forward) / grad_out (backward)
    void *gread, *ggate;
    long ggate_stride;
    float *partial;    // [CTAs][HD]
};

// Thread = one (token, head) row; consecutive threads are consecutive heads
// of a token, so gate and output rows are contiguous across a warp and each
// read row is one 32-byte-aligned segment.
template <bool RBF, bool GBF, int HD>
__global__ void __launch_bounds__(kThreads) epilogue_kernel(const EpiArgs a) {
    const long row = static_cast<long>(blockIdx.x) * kThreads + threadIdx.x;
    const long rows = a.b * a.t * a.heads;
    if (row >= rows) return;
    const long tok = row / a.heads;  // b * T + t
    const int h = static_cast<int>(row - tok * a.heads);
    const long bb = tok / a.t, t = tok - bb * a.t;
    float r[HD], g[HD];
    ldv<RBF, HD>(a.read, ((bb * a.heads + h) * a.t + t) * HD, r);
    ldv<GBF, HD>(a.gate, tok * a.gate_stride + static_cast<long>(h) * HD, g);
    float ms = 0.f;
#pragma unroll
    for (int i = 0; i < HD; ++i) {
        if constexpr (GBF) r[i] = round_bf16(r[i]);  // read.to(x.dtype)
        ms = fmaf(r[i], r[i], ms);
    }
    const float inv = rsqrtf(ms * (1.0f / HD) + a.eps);
    float o[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] = r[i] * inv * __ldg(a.w + i) * (g[i] * sigmoid(g[i]));
    stv<GBF, HD>(a.out, tok * static_cast<long>(a.heads) * HD + static_cast<long>(h) * HD, o);
}

template <bool RBF, bool GBF, int HD>
__global__ void __launch_bounds__(kThreads) epilogue_backward_kernel(const EpiArgs a) {
    __shared__ float red[kThreads / 32][HD];
    const long row = static_cast<long>(blockIdx.x) * kThreads + threadIdx.x;
    const long rows = a.b * a.t * a.heads;
    float gw[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) gw[i] = 0.f;
    if (row < rows) {
        const long tok = row / a.heads;
        const int h = static_cast<int>(row - tok * a.heads);
        const long bb = tok / a.t, t = tok - bb * a.t;
        const long rix = ((bb * a.heads + h) * a.t + t) * HD;
        float r[HD], g[HD], go[HD], w[HD];
        ldv<RBF, HD>(a.read, rix, r);
        ldv<GBF, HD>(a.gate, tok * a.gate_stride + static_cast<long>(h) * HD, g);
        ldv<GBF, HD>(a.out, tok * static_cast<long>(a.heads) * HD + static_cast<long>(h) * HD, go);
        float ms = 0.f;
#pragma unroll
        for (int i = 0; i < HD; ++i) {
            if constexpr (GBF) r[i] = round_bf16(r[i]);
            w[i] = __ldg(a.w + i);
            ms = fmaf(r[i], r[i], ms);
        }
        const float inv = rsqrtf(ms * (1.0f / HD) + a.eps);
        float ggt[HD], gr[HD], dot = 0.f;
#pragma unroll
        for (int i = 0; i < HD; ++i) {
            const float sg = sigmoid(g[i]);
            const float silu = g[i] * sg, dsilu = sg * fmaf(g[i], 1.f - sg, 1.f);
            const float n = r[i] * inv;            // normalised, before the weight
            ggt[i] = go[i] * n * w[i] * dsilu;     // d/dgate
            const float gy = go[i] * silu;         // d/d(normalised * weight)
            gw[i] = gy * n;
            gr[i] = w[i] * gy;                     // z = w * gy
            dot = fmaf(r[i], gr[i], dot);
        }
        // d/dr of r * inv: inv * z - r * inv^3 * (r . z) / HD
        const float c3 = inv * inv * inv * dot * (1.0f / HD);
#pragma unroll
        for (int i = 0; i < HD; ++i) gr[i] = inv * gr[i] - r[i] * c3;
        stv<RBF, HD>(a.gread, rix, gr);
        stv<GBF, HD>(a.ggate, tok * a.ggate_stride + static_cast<long>(h) * HD, ggt);
    }
    // weight gradient: warp sums, then the CTA's warps in order
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < HD; ++i) {
        float v = gw[i];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) red[warp][i] = v;
    }
    __syncthreads();
    if (threadIdx.x < HD) {
        float acc = 0.f;
#pragma unroll
        for (int wv = 0; wv < kThreads / 32; ++wv) acc += red[wv][threadIdx.x];
        a.partial[static_cast<long>(blockIdx.x) * HD + threadIdx.x] = acc;
    }
}

// Tiled readout for head dims 8 and 16, where a (token, head) row of the
// chain-major reads is only 32 or 64 bytes and the row-per-thread kernels
// above touch one scattered sector per thread.  A CTA takes 32 heads x (256 /
// HD) tokens of one batch row: it copies each head's run of tokens (256
// contiguous elements) into a shared tile, then works the rows in token-major
// order, so the gate, output and gate-gradient rows of a warp are contiguous
// too.  The backward writes the read gradient back through the same tile.
template <int HD>
struct EpiTile {
    static constexpr int kT = 256 / HD;        // tokens per tile
    static constexpr int kH = 32;              // heads per tile
    static constexpr int kRowF = kT * HD + 4;  // floats per head in shared memory (+4: float4 reads across heads hit distinct banks)
};

inline long epi_tiles(long b, long t, int heads, int hd) {
    return b * ((t + 256 / hd - 1) / (256 / hd)) * ((heads + 31) / 32);
}

template <int HD>
__device__ __forceinline__ void epi_tile_of(const EpiArgs &a, long &bb, long &t0, int &h0) {
    constexpr int kT = EpiTile<HD>::kT;
    const long ht = (a.heads + 31) / 32, tt = (a.t + kT - 1) / kT;
    long i = blockIdx.x;
    h0 = static_cast<int>(i % ht) * 32;
    i /= ht;
    t0 = (i % tt) * kT;
    bb = i / tt;
}

// Four elements per thread and head, 64 threads per head: heads hl, hl + 4, ...
// Elements past the sequence end or past the last head stay zero in the tile.
template <bool RBF, int HD>
__device__ __forceinline__ void epi_load_tile(const EpiArgs &a, long bb, long t0, int h0,
                                              float (*sm)[EpiTile<HD>::kRowF]) {
    constexpr int kT = EpiTile<HD>::kT;
    const int valid = static_cast<int>((a.t - t0 < kT ? a.t - t0 : kT) * HD);
    const int e = (threadIdx.x & 63) * 4;
    for (int hl = threadIdx.x >> 6; hl < EpiTile<HD>::kH; hl += kThreads / 64) {
        const int h = h0 + hl;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (h < a.heads && e < valid) ldn<RBF, 4>(a.read, ((bb * a.heads + h) * a.t + t0) * HD + e, v);
        *reinterpret_cast<float4 *>(&sm[hl][e]) = make_float4(v[0], v[1], v[2], v[3]);
    }
}

template <bool RBF, bool GBF, int HD>
__global__ void __launch_bounds__(kThreads) epilogue_tile_kernel(const EpiArgs a) {
    using E = EpiTile<HD>;
    __shared__ __align__(16) float sm[E::kH][E::kRowF];
    long bb, t0;
    int h0;
    epi_tile_of<HD>(a, bb, t0, h0);
    epi_load_tile<RBF, HD>(a, bb, t0, h0, sm);
    __syncthreads();
    const int hl = threadIdx.x & 31, h = h0 + hl;
    float w[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) w[i] = __ldg(a.w + i);
    for (int tl = threadIdx.x >> 5; tl < E::kT; tl += kThreads / 32) {
        const long t = t0 + tl;
        if (h >= a.heads || t >= a.t) continue;
        const long tok = bb * a.t + t;
        float r[HD], g[HD];
#pragma unroll
        for (int i = 0; i < HD; i += 4) {
            const float4 f = *reinterpret_cast<const float4 *>(&sm[hl][tl * HD + i]);
            r[i] = f.x, r[i + 1] = f.y, r[i + 2] = f.z, r[i + 3] = f.w;
        }
        ldv<GBF, HD>(a.gate, tok * a.gate_stride + static_cast<long>(h) * HD, g);
        float ms = 0.f;
#pragma unroll
        for (int i = 0; i < HD; ++i) {
            if constexpr (GBF) r[i] = round_bf16(r[i]);  // read.to(x.dtype)
            ms = fmaf(r[i], r[i], ms);
        }
        const float inv = rsqrtf(ms * (1.0f / HD) + a.eps);
        float o[HD];
#pragma unroll
        for (int i = 0; i < HD; ++i) o[i] = r[i] * inv * w[i] * (g[i] * sigmoid(g[i]));
        stv<GBF, HD>(a.out, tok * static_cast<long>(a.heads) * HD + static_cast<long>(h) * HD, o);
    }
}

template <bool RBF, bool GBF, int HD>
__global__ void __launch_bounds__(kThreads) epilogue_tile_backward_kernel(const EpiArgs a) {
    using E = EpiTile<HD>;
    __shared__ __align__(16) float sm[E::kH][E::kRowF];
    __shared__ float red[kThreads / 32][HD];
    long bb, t0;
    int h0;
    epi_tile_of<HD>(a, bb, t0, h0);
    epi_load_tile<RBF, HD>(a, bb, t0, h0, sm);
    __syncthreads();
    const int hl = threadIdx.x & 31, h = h0 + hl;
    float w[HD], gw[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) {
        w[i] = __ldg(a.w + i);
        gw[i] = 0.f;
    }
#pragma unroll  // later rows' gate and output-gradient loads issue early (forward: no gain, 0.126 vs 0.119 ms)
    for (int tl = threadIdx.x >> 5; tl < E::kT; tl += kThreads / 32) {
        const long t = t0 + tl;
        if (h >= a.heads || t >= a.t) continue;
        const long tok = bb * a.t + t;
        float r[HD], g[HD], go[HD];
#pragma unroll
        for (int i = 0; i < HD; i += 4) {
            const float4 f = *reinterpret_cast<const float4 *>(&sm[hl][tl * HD + i]);
            r[i] = f.x, r[i + 1] = f.y, r[i + 2] = f.z, r[i + 3] = f.w;
        }
        ldv<GBF, HD>(a.gate, tok * a.gate_stride + static_cast<long>(h) * HD, g);
        ldv<GBF, HD>(a.out, tok * static_cast<long>(a.heads) * HD + static_cast<long>(h) * HD, go);
        float ms = 0.f;
#pragma unroll
        for (int i = 0; i < HD; ++i) {
            if constexpr (GBF) r[i] = round_bf16(r[i]);
            ms = fmaf(r[i], r[i], ms);
        }
        const float inv = rsqrtf(ms * (1.0f / HD) + a.eps);
        float ggt[HD], gr[HD], dot = 0.f;
#pragma unroll
        for (int i = 0; i < HD; ++i) {
            const float sg = sigmoid(g[i]);
            const float silu = g[i] * sg, dsilu = sg * fmaf(g[i], 1.f - sg, 1.f);
            const float n = r[i] * inv;          // normalised, before the weight
            ggt[i] = go[i] * n * w[i] * dsilu;   // d/dgate
            const float gy = go[i] * silu;       // d/d(normalised * weight)
            gw[i] = fmaf(gy, n, gw[i]);
            gr[i] = w[i] * gy;                   // z = w * gy
            dot = fmaf(r[i], gr[i], dot);
        }
        // d/dr of r * inv: inv * z - r * inv^3 * (r . z) / HD
        const float c3 = inv * inv * inv * dot * (1.0f / HD);
#pragma unroll
        for (int i = 0; i < HD; ++i) gr[i] = inv * gr[i] - r[i] * c3;
        stv<GBF, HD>(a.ggate, tok * a.ggate_stride + static_cast<long>(h) * HD, ggt);
#pragma unroll
        for (int i = 0; i < HD; i += 4)  // this thread's own row of the tile
            *reinterpret_cast<float4 *>(&sm[hl][tl * HD + i]) = make_float4(gr[i], gr[i + 1], gr[i + 2], gr[i + 3]);
    }
    __syncthreads();
    {  // the read gradient, each head's run of tokens as one contiguous store
        constexpr int kT = E::kT;
        const int valid = static_cast<int>((a.t - t0 < kT ? a.t - t0 : kT) * HD);
        const int e = (threadIdx.x & 63) * 4;
        for (int hx = threadIdx.x >> 6; hx < E::kH; hx += kThreads / 64) {
            const int hh = h0 + hx;
            if (hh < a.heads && e < valid) {
                const float4 f = *reinterpret_cast<const float4 *>(&sm[hx][e]);
                const float v[4] = {f.x, f.y, f.z, f.w};
                stn<RBF, 4>(a.gread, ((bb * a.heads + hh) * a.t + t0) * HD + e, v);
            }
        }
    }
    // weight gradient: warp sums, then the CTA's warps in order
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < HD; ++i) {
        float v = gw[i];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) red[warp][i] = v;
    }
    __syncthreads();
    if (threadIdx.x < HD) {
        float acc = 0.f;
#pragma unroll
        for (int wv = 0; wv < kThreads / 32; ++wv) acc += red[wv][threadIdx.x];
        a.partial[static_cast<long>(blockIdx.x) * HD + threadIdx.x] = acc;
    }
}

// First pass of the many-column sum: CTA (x, y) sums rows [y * per, (y + 1) *
// per) of its columns into row y of `out` (rows in order).
__global__ void __launch_bounds__(kThreads) reduce_row_groups_kernel(const float *partial, long rows, int cols,
                                                                     int stride, long per, float *out) {
    const int e = static_cast<int>(blockIdx.x) * kThreads + threadIdx.x;
    if (e >= cols) return;
    const long r0 = static_cast<long>(blockIdx.y) * per;
    const long r1 = r0 + per < rows ? r0 + per : rows;
    float acc = 0.f;
#pragma unroll 8
    for (long r = r0; r < r1; ++r) acc += partial[r * stride + e];
    out[static_cast<long>(blockIdx.y) * stride + e] = acc;
}

// ---- input RMSNorm (nn.RMSNorm over the width, the mixer's first op) -------
// A warp owns a row; lane l holds chunks c * 32 + l of 8 elements (each chunk
// index is one 16-byte vector), so every load and store is coalesced.
constexpr int kNormRowsPerCta = kThreads / 32;

template <bool BF, int CPL>
__global__ void __launch_bounds__(kThreads) rmsnorm_kernel(const void *x, const float *w, void *out, long rows,
                                                          float eps) {
    constexpr int W = 256 * CPL;
    const int lane = threadIdx.x & 31;
    const long row = static_cast<long>(blockIdx.x) * kNormRowsPerCta + (threadIdx.x >> 5);
    if (row >= rows) return;  // whole warps
    float v[8 * CPL];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        ldn<BF, 8>(x, row * W + (c * 32 + lane) * 8, v + 8 * c);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(v[8 * c + i], v[8 * c + i], ss);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = rsqrtf(ss * (1.0f / W) + eps);
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        float wv[8];
        ldn<false, 8>(w, (c * 32 + lane) * 8, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[8 * c + i] = v[8 * c + i] * inv * wv[i];
        stn<BF, 8>(out, row * W + (c * 32 + lane) * 8, v + 8 * c);
    }
}

// Backward: gx = inv (w gy) - x inv^3 (x . w gy) / W per row; the weight
// gradient sum_rows gy x inv is kept per lane over the rows a warp visits
// (grid-stride), then summed over the CTA's warps in order into one partial
// row per CTA.
template <bool BF, int CPL>
__global__ void __launch_bounds__(kThreads) rmsnorm_backward_kernel(const void *x, const float *w, const void *gy,
                                                                   void *gx, long rows, float eps, float *partial) {
    constexpr int W = 256 * CPL;
    __shared__ float red[kNormRowsPerCta][W];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float wv[8 * CPL], gw[8 * CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) ldn<false, 8>(w, (c * 32 + lane) * 8, wv + 8 * c);
#pragma unroll
    for (int i = 0; i < 8 * CPL; ++i) gw[i] = 0.f;
    for (long row = static_cast<long>(blockIdx.x) * kNormRowsPerCta + warp; row < rows;
         row += static_cast<long>(gridDim.x) * kNormRowsPerCta) {
        float xv[8 * CPL], g[8 * CPL];
        float ss = 0.f, dot = 0.f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            ldn<BF, 8>(x, row * W + (c * 32 + lane) * 8, xv + 8 * c);
            ldn<BF, 8>(gy, row * W + (c * 32 + lane) * 8, g + 8 * c);
        }
#pragma unroll
        for (int i = 0; i < 8 * CPL; ++i) ss = fmaf(xv[i], xv[i], ss);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        const float inv = rsqrtf(ss * (1.0f / W) + eps);
#pragma unroll
        for (int i = 0; i < 8 * CPL; ++i) {
            gw[i] = fmaf(g[i] * xv[i], inv, gw[i]);  // gy x inv
            g[i] *= wv[i];                           // z = w gy
            dot = fmaf(xv[i], g[i], dot);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        const float c3 = inv * inv * inv * dot * (1.0f / W);
#pragma unroll
        for (int i = 0; i < 8 * CPL; ++i) g[i] = inv * g[i] - xv[i] * c3;
#pragma unroll
        for (int c = 0; c < CPL; ++c) stn<BF, 8>(gx, row * W + (c * 32 + lane) * 8, g + 8 * c);
    }
#pragma unroll
    for (int c = 0; c < CPL; ++c)
#pragma unroll
        for (int i = 0; i < 8; ++i) red[warp][(c * 32 + lane) * 8 + i] = gw[8 * c + i];
    __syncthreads();
    for (int e = threadIdx.x; e < W; e += kThreads) {
        float acc = 0.f;
#pragma unroll
        for (int wp = 0; wp < kNormRowsPerCta; ++wp) acc += red[wp][e];
        partial[static_cast<long>(blockIdx.x) * W + e] = acc;
    }
}

// out[e] = sum over r of partial[r][e], rows in order (deterministic).
__global__ void __launch_bounds__(kThreads) reduce_rows_kernel(const float *partial, long rows, int cols, int stride,
                                                               float *gw, int nw, float *gbias) {
    const int e = static_cast<int>(blockIdx.x) * kThreads + threadIdx.x;
    if (e >= cols) return;
    float acc = 0.f;
    for (long r = 0; r < rows; ++r) acc += partial[r * stride + e];
    if (e < nw) {
        gw[e] = acc;
    } else if (gbias != nullptr) {
        gbias[e - nw] = acc;
    }
}

// The same for few columns and many rows: CTA e sums column e, thread i
// taking rows i, i + 256, ... in order, then a fixed-shape tree over threads.
__global__ void __launch_bounds__(kThreads) reduce_cols_kernel(const float *partial, long rows, int stride,
                                                               float *out) {
    __shared__ float red[kThreads];
    const int e = blockIdx.x;
    float acc = 0.f;
    for (long r = threadIdx.x; r < rows; r += kThreads) acc += partial[r * stride + e];
    red[threadIdx.x] = acc;
    __syncthreads();
    for (int half = kThreads / 2; half > 0; half >>= 1) {
        if (threadIdx.x < half) red[threadIdx.x] += red[threadIdx.x + half];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[e] = red[0];
}

int check_shape(const Shape &s, int in_dtype, int out_dtype) {
    if (s.b < 0 || s.t < 0 || s.heads <= 0 || s.hd <= 0 || s.d <= 0)
        return fail(BSSM_ERR_INVALID, "envelope: bad sizes");
    if (s.d < 2 || s.d > 64 || (s.d & (s.d - 1)) != 0 || (s.hd & 1))
        return fail(BSSM_ERR_UNSUPPORTED, "envelope: key_dim must be a power of two in [2, 64] and head_dim even "
                    "(got %d, %d)", s.d, s.hd);
    if ((in_dtype != BSSM_F32 && in_dtype != BSSM_BF16) || (out_dtype != BSSM_F32 && out_dtype != BSSM_BF16))
        return fail(BSSM_ERR_UNSUPPORTED, "envelope: dtypes must be float32 or bfloat16");
    if (s.in_stride < s.conv_channels() + s.aux_channels() || (s.in_stride & 1))
        return fail(BSSM_ERR_INVALID, "envelope: projection row stride %ld is odd or shorter than %d channels",
                    s.in_stride, s.conv_channels() + s.aux_channels());
    if (s.b > 65535) return fail(BSSM_ERR_INVALID, "envelope: at most 65535 batch rows per call");
    return BSSM_OK;
}

// Channel-group width CW: every stream and head row boundary must fall on a
// multiple of CW, and the vector accesses of CW >= 4 need 16-byte aligned
// tensors.
template <int CW>
bool cw_fits(const Shape &s, long other_stride, const void *const *ptrs, int nptr) {
    if (s.sw() % CW || s.hd % CW || (2 * s.heads) % CW || s.in_stride % CW || other_stride % CW) return false;
    if (CW >= 4)
        for (int i = 0; i < nptr; ++i)
            if (reinterpret_cast<uintptr_t>(ptrs[i]) & 15) return false;
    return true;
}

// One warp per 32 channel groups of each (batch row, span); see work_of.
bool too_many_ctas(const Shape &s) {  // two channels per thread launch the most
    const long wpr = ((s.conv_channels() + s.aux_channels()) / 2 + 31) / 32;
    return (s.b * s.tsplit * wpr + kThreads / 32 - 1) / (kThreads / 32) > 0x7fffffffL;
}
template <int CW>
dim3 grid_of(const Shape &s) {
    const long wpr = ((s.conv_channels() + s.aux_channels()) / CW + 31) / 32;
    const long warps = s.b * s.tsplit * wpr;
    return dim3(static_cast<unsigned>((warps + kThreads / 32 - 1) / (kThreads / 32)));
}

template <int CW, int L>
void launch_fwd(const Shape &s, const ProArgs &a, int in_dtype, int out_dtype, cudaStream_t st) {
    const dim3 g = grid_of<CW>(s);
    if (in_dtype == BSSM_BF16) {
        if (out_dtype == BSSM_BF16) prologue_kernel<true, true, CW, L><<<g, kThreads, 0, st>>>(s, a);
        else prologue_kernel<true, false, CW, L><<<g, kThreads, 0, st>>>(s, a);
    } else {
        if (out_dtype == BSSM_BF16) prologue_kernel<false, true, CW, L><<<g, kThreads, 0, st>>>(s, a);
        else prologue_kernel<false, false, CW, L><<<g, kThreads, 0, st>>>(s, a);
    }
}

template <int CW, int L>
void launch_bwd(const Shape &s, const EnvBwdArgs &a, int in_dtype, int out_dtype, cudaStream_t st) {
    const dim3 g = grid_of<CW>(s);
    if (in_dtype == BSSM_BF16) {
        if (out_dtype == BSSM_BF16) prologue_backward_kernel<true, true, CW, L><<<g, kThreads, 0, st>>>(s, a);
        else prologue_backward_kernel<true, false, CW, L><<<g, kThreads, 0, st>>>(s, a);
    } else {
        if (out_dtype == BSSM_BF16) prologue_backward_kernel<false, true, CW, L><<<g, kThreads, 0, st>>>(s, a);
        else prologue_backward_kernel<false, false, CW, L><<<g, kThreads, 0, st>>>(s, a);
    }
}

// Four channels per thread where the shape allows it (a thread then never
// holds more than one q / k head: key dim >= 4), else two; the lanes per head
// fixed at compile time for the common key dims.
void dispatch_bwd(const Shape &s, const EnvBwdArgs &a, const void *const *aligned, int nal, int in_dtype,
                  int out_dtype, cudaStream_t st) {
    if (kBwdCW >= 4 && s.d >= 4 && cw_fits<4>(s, a.gx_stride, aligned, nal)) {
        if (s.d == 4) launch_bwd<4, 1>(s, a, in_dtype, out_dtype, st);
        else if (s.d == 8) launch_bwd<4, 2>(s, a, in_dtype, out_dtype, st);
        else launch_bwd<4, 0>(s, a, in_dtype, out_dtype, st);
    } else {
        if (s.d == 2) launch_bwd<2, 1>(s, a, in_dtype, out_dtype, st);
        else if (s.d == 4) launch_bwd<2, 2>(s, a, in_dtype, out_dtype, st);
        else if (s.d == 8) launch_bwd<2, 4>(s, a, in_dtype, out_dtype, st);
        else launch_bwd<2, 0>(s, a, in_dtype, out_dtype, st);
    }
}

int pick_tsplit(long t, int span) { return static_cast<int>((t + span - 1) / span); }

int epi_check(long batch, long tokens, int heads, int head_dim, int read_dtype, int gate_dtype, long gate_stride) {
    if (batch < 0 || tokens < 0 || heads <= 0) return fail(BSSM_ERR_INVALID, "envelope epilogue: bad sizes");
    if (head_dim != 8 && head_dim != 16 && head_dim != 32 && head_dim != 64)
        return fail(BSSM_ERR_UNSUPPORTED, "envelope epilogue: head_dim must be 8, 16, 32 or 64 (got %d)", head_dim);
    if ((read_dtype != BSSM_F32 && read_dtype != BSSM_BF16) || (gate_dtype != BSSM_F32 && gate_dtype != BSSM_BF16))
        return fail(BSSM_ERR_UNSUPPORTED, "envelope epilogue: dtypes must be float32 or bfloat16");
    if (gate_stride < static_cast<long>(heads) * head_dim || gate_stride % 8)
        return fail(BSSM_ERR_INVALID, "envelope epilogue: gate row stride %ld is short or not a multiple of 8",
                    gate_stride);
    return BSSM_OK;
}

// CTAs the readout launches for a shape (tiles for head dims 8 and 16, else
// one CTA per 256 rows); the backward writes one partial-sum row per CTA.
long epi_ctas(long b, long t, int heads, int hd) {
    if (hd == 8 || hd == 16) return epi_tiles(b, t, heads, hd);
    return (b * t * heads + kThreads - 1) / kThreads;
}

template <int HD>
void launch_epi(const EpiArgs &a, int rd, int gd, bool backward, cudaStream_t st) {
    const unsigned grid = static_cast<unsigned>(epi_ctas(a.b, a.t, a.heads, HD));
#define BSSM_EPI(R, G)                                                                            \
    do {                                                                                          \
        if constexpr (HD == 8 || HD == 16) {                                                      \
            if (backward) epilogue_tile_backward_kernel<R, G, HD><<<grid, kThreads, 0, st>>>(a); \
            else epilogue_tile_kernel<R, G, HD><<<grid, kThreads, 0, st>>>(a);                   \
        } else {                                                                                  \
            if (backward) epilogue_backward_kernel<R, G, HD><<<grid, kThreads, 0, st>>>(a);      \
            else epilogue_kernel<R, G, HD><<<grid, kThreads, 0, st>>>(a);                        \
        }                                                                                         \
    } while (0)
    if (rd == BSSM_BF16) {
        if (gd == BSSM_BF16) BSSM_EPI(true, true);
        else BSSM_EPI(true, false);
    } else {
        if (gd == BSSM_BF16) BSSM_EPI(false, true);
        else BSSM_EPI(false, false);
    }
#undef BSSM_EPI
}

void launch_epi_hd(const EpiArgs &a, int hd, int rd, int gd, bool backward, cudaStream_t st) {
    switch (hd) {
        case 8: launch_epi<8>(a, rd, gd, backward, st); break;
        case 16: launch_epi<16>(a, rd, gd, backward, st); break;
        case 32: launch_epi<32>(a, rd, gd, backward, st); break;
        default: launch_epi<64>(a, rd, gd, backward, st); break;
    }
}

template <int CPL>
void launch_norm(const void *x, int dt, const float *w, const void *gy, void *out, long rows, float eps,
                 float *partial, int ctas, cudaStream_t st) {
    if (gy == nullptr) {
        const unsigned grid = static_cast<unsigned>((rows + kNormRowsPerCta - 1) / kNormRowsPerCta);
        if (dt == BSSM_BF16) rmsnorm_kernel<true, CPL><<<grid, kThreads, 0, st>>>(x, w, out, rows, eps);
        else rmsnorm_kernel<false, CPL><<<grid, kThreads, 0, st>>>(x, w, out, rows, eps);
    } else {
        if (dt == BSSM_BF16) rmsnorm_backward_kernel<true, CPL><<<ctas, kThreads, 0, st>>>(x, w, gy, out, rows, eps, partial);
        else rmsnorm_backward_kernel<false, CPL><<<ctas, kThreads, 0, st>>>(x, w, gy, out, rows, eps, partial);
    }
}

// Backward grid: one full wave (resident CTAs per SM x SMs), at most `cap`.
// The wave is queried once per device and dtype, then cached.
template <int CPL>
int norm_wave(int dt, int cap) {
    constexpr int kMaxDevices = 64;
    static std::atomic<int> cached[kMaxDevices][2];  // 0: not queried yet
    int dev = 0, sms = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cap;
    const int bf = dt == BSSM_BF16 ? 1 : 0;
    int wave = dev >= 0 && dev < kMaxDevices ? cached[dev][bf].load(std::memory_order_relaxed) : 0;
    if (wave == 0) {
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return cap;
        const cudaError_t err =
            bf ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rmsnorm_backward_kernel<true, CPL>, kThreads, 0)
               : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rmsnorm_backward_kernel<false, CPL>, kThreads, 0);
        if (err != cudaSuccess || per_sm <= 0) return cap;
        const long w = static_cast<long>(per_sm) * sms;
        wave = static_cast<int>(w < 0x7fffffffL ? w : 0x7fffffffL);
        if (dev >= 0 && dev < kMaxDevices) cached[dev][bf].store(wave, std::memory_order_relaxed);
    }
    return wave < cap ? wave : cap;
}

int norm_wave_w(int width, int dt, int cap) {
    switch (width / 256) {
        case 1: return norm_wave<1>(dt, cap);
        case 2: return norm_wave<2>(dt, cap);
        case 3: return norm_wave<3>(dt, cap);
        default: return norm_wave<4>(dt, cap);
    }
}

void launch_norm_w(int width, const void *x, int dt, const float *w, const void *gy, void *out, long rows, float eps,
                   float *partial, int ctas, cudaStream_t st) {
    switch (width / 256) {
        case 1: launch_norm<1>(x, dt, w, gy, out, rows, eps, partial, ctas, st); break;
        case 2: launch_norm<2>(x, dt, w, gy, out, rows, eps, partial, ctas, st); break;
        case 3: launch_norm<3>(x, dt, w, gy, out, rows, eps, partial, ctas, st); break;
        default: launch_norm<4>(x, dt, w, gy, out, rows, eps, partial, ctas, st); break;
    }
}

constexpr int kNormCtas = 4 * 148;  // most backward CTAs (grid-stride over rows); sizes the workspace

int norm_check(long rows, int width, int dtype) {
    if (rows < 0) return fail(BSSM_ERR_INVALID, "rms_norm: negative rows");
    if (width <= 0 || width % 256 || width > 1024)
        return fail(BSSM_ERR_UNSUPPORTED, "rms_norm: width must be 256, 512, 768 or 1024 (got %d)", width);
    if (dtype != BSSM_F32 && dtype != BSSM_BF16) return fail(BSSM_ERR_UNSUPPORTED, "rms_norm: float32 or bfloat16");
    return BSSM_OK;
}

}  // namespace env
}  // namespace bssm

using namespace bssm;
using namespace bssm::env;

extern "C" {

long bssm_envelope_partial_floats(long batch, long tokens, int heads, int key_dim, int head_dim) {
    Shape s{batch, tokens, heads, key_dim, head_dim, 0, 1};
    // per-span partial rows, then the row-group sums of the first reduction pass
    return (batch * pick_tsplit(tokens, kBwdSpan) + kRowGroups) * static_cast<long>(s.partial_cols());
}

int bssm_envelope_prologue(const void *projected, int in_dtype, long batch, long tokens, int heads, int key_dim,
                           int head_dim, long row_stride, const float *conv_weight, const float *aux_bias,
                           void *keys, void *queries, void *values, int out_dtype, float *decay, float *process,
                           float *observation, unsigned *check_flags, void *stream) {
    Shape s{batch, tokens, heads, key_dim, head_dim, row_stride, 1};
    if (int rc = check_shape(s, in_dtype, out_dtype)) return rc;
    if (batch == 0 || tokens == 0) {
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!projected || !conv_weight || !keys || !queries || !values || !decay || !process || !observation)
        return fail(BSSM_ERR_INVALID, "envelope prologue: null pointer");
    const void *aligned8[] = {projected, keys, queries, values, decay};
    for (const void *p : aligned8)
        if (reinterpret_cast<uintptr_t>(p) & 7)
            return fail(BSSM_ERR_ALIGNMENT, "envelope prologue: tensors must be 8-byte aligned");
    if (reinterpret_cast<uintptr_t>(conv_weight) & 15)
        return fail(BSSM_ERR_ALIGNMENT, "envelope prologue: conv_weight must be 16-byte aligned");
    s.tsplit = pick_tsplit(tokens, kFwdSpan);
    if (s.tsplit > 65535 || too_many_ctas(s))
        return fail(BSSM_ERR_INVALID, "envelope: sequence too long (%ld tokens)", tokens);
    if (check_flags != nullptr && (reinterpret_cast<uintptr_t>(check_flags) & 3))
        return fail(BSSM_ERR_ALIGNMENT, "envelope prologue: check_flags must be 4-byte aligned");
    const ProArgs a{projected, conv_weight, aux_bias, keys, queries, values, decay, process, observation,
                    check_flags};
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (kFwdCW >= 4 && cw_fits<4>(s, 0, aligned8, 5)) {
        if (s.d == 4) launch_fwd<4, 1>(s, a, in_dtype, out_dtype, st);
        else if (s.d == 8) launch_fwd<4, 2>(s, a, in_dtype, out_dtype, st);
        else launch_fwd<4, 0>(s, a, in_dtype, out_dtype, st);
    } else {
        launch_fwd<2, 0>(s, a, in_dtype, out_dtype, st);
    }
    return check_launch("envelope prologue");
}

int bssm_envelope_prologue_backward(const void *projected, int in_dtype, long batch, long tokens, int heads,
                                    int key_dim, int head_dim, long row_stride, const float *conv_weight,
                                    const float *aux_bias, const void *grad_keys, const void *grad_queries,
                                    const void *grad_values, int out_dtype, const float *grad_decay,
                                    const float *grad_process, const float *grad_observation, void *grad_projected,
                                    long grad_row_stride, float *grad_conv_weight, float *grad_aux_bias,
                                    float *workspace, long workspace_floats, void *stream) {
    Shape s{batch, tokens, heads, key_dim, head_dim, row_stride, 1};
    if (int rc = check_shape(s, in_dtype, out_dtype)) return rc;
    if (grad_row_stride < s.conv_channels() + s.aux_channels() || (grad_row_stride & 1))
        return fail(BSSM_ERR_INVALID, "envelope backward: gradient row stride %ld is odd or too short",
                    grad_row_stride);
    if (!grad_conv_weight) return fail(BSSM_ERR_INVALID, "envelope backward: null weight gradient");
    const int C = s.conv_channels(), cols = 4 * C + s.aux_channels(), pcols = s.partial_cols();
    if (batch == 0 || tokens == 0) {
        cudaError_t err = cudaMemsetAsync(grad_conv_weight, 0, sizeof(float) * 4 * C, static_cast<cudaStream_t>(stream));
        if (err == cudaSuccess && grad_aux_bias)
            err = cudaMemsetAsync(grad_aux_bias, 0, sizeof(float) * s.aux_channels(), static_cast<cudaStream_t>(stream));
        if (err != cudaSuccess) return fail(BSSM_ERR_CUDA, "envelope backward: %s", cudaGetErrorString(err));
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!projected || !conv_weight || !grad_projected || !workspace)
        return fail(BSSM_ERR_INVALID, "envelope backward: null pointer");
    s.tsplit = pick_tsplit(tokens, kBwdSpan);
    if (s.tsplit > 65535 || too_many_ctas(s))
        return fail(BSSM_ERR_INVALID, "envelope: sequence too long (%ld tokens)", tokens);
    const long prow = batch * s.tsplit;
    const long need = (prow + kRowGroups) * static_cast<long>(pcols);
    if (workspace_floats < need)
        return fail(BSSM_ERR_WORKSPACE, "envelope backward: workspace of %ld floats, need %ld", workspace_floats, need);
    if (reinterpret_cast<uintptr_t>(workspace) & 31)
        return fail(BSSM_ERR_ALIGNMENT, "envelope backward: workspace must be 32-byte aligned");
    const void *aligned8[] = {projected, grad_projected, grad_keys, grad_queries, grad_values, grad_decay};
    for (const void *p : aligned8)
        if (reinterpret_cast<uintptr_t>(p) & 7)
            return fail(BSSM_ERR_ALIGNMENT, "envelope backward: tensors must be 8-byte aligned");
    if (reinterpret_cast<uintptr_t>(conv_weight) & 15)
        return fail(BSSM_ERR_ALIGNMENT, "envelope backward: conv_weight must be 16-byte aligned");
    const EnvBwdArgs a{projected, conv_weight, aux_bias, grad_keys, grad_queries, grad_values, grad_decay, grad_process,
                    grad_observation, grad_projected, grad_row_stride, workspace};
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    dispatch_bwd(s, a, aligned8, 6, in_dtype, out_dtype, st);
    if (int rc = check_launch("envelope prologue backward")) return rc;
    // two passes, each summing rows in order: row groups, then the groups
    const long per = (prow + kRowGroups - 1) / kRowGroups;
    const int groups = static_cast<int>((prow + per - 1) / per);
    float *const sums = workspace + prow * pcols;
    reduce_row_groups_kernel<<<dim3((cols + kThreads - 1) / kThreads, groups), kThreads, 0, st>>>(
        workspace, prow, cols, pcols, per, sums);
    if (int rc = check_launch("envelope reduction")) return rc;
    reduce_rows_kernel<<<(cols + kThreads - 1) / kThreads, kThreads, 0, st>>>(sums, groups, cols, pcols,
                                                                               grad_conv_weight, 4 * C, grad_aux_bias);
    return check_launch("envelope reduction");
}

long bssm_rms_norm_partial_floats(long rows, int width) {
    (void)rows;
    return static_cast<long>(kNormCtas + kRowGroups) * width;
}

int bssm_rms_norm(const void *x, int dtype, long rows, int width, const float *weight, float eps, void *out,
                  void *stream) {
    if (int rc = norm_check(rows, width, dtype)) return rc;
    if (rows == 0) {
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!x || !weight || !out) return fail(BSSM_ERR_INVALID, "rms_norm: null pointer");
    const void *al[] = {x, weight, out};
    for (const void *p : al)
        if (reinterpret_cast<uintptr_t>(p) & 15) return fail(BSSM_ERR_ALIGNMENT, "rms_norm: tensors must be 16-byte aligned");
    launch_norm_w(width, x, dtype, weight, nullptr, out, rows, eps, nullptr, 0, static_cast<cudaStream_t>(stream));
    return check_launch("rms_norm");
}

int bssm_rms_norm_backward(const void *x, int dtype, long rows, int width, const float *weight, float eps,
                           const void *grad_out, void *grad_x, float *grad_weight, float *workspace,
                           long workspace_floats, void *stream) {
    if (int rc = norm_check(rows, width, dtype)) return rc;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!grad_weight) return fail(BSSM_ERR_INVALID, "rms_norm backward: null weight gradient");
    if (rows == 0) {
        const cudaError_t err = cudaMemsetAsync(grad_weight, 0, sizeof(float) * width, st);
        if (err != cudaSuccess) return fail(BSSM_ERR_CUDA, "rms_norm backward: %s", cudaGetErrorString(err));
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!x || !weight || !grad_out || !grad_x || !workspace) return fail(BSSM_ERR_INVALID, "rms_norm backward: null pointer");
    if (workspace_floats < bssm_rms_norm_partial_floats(rows, width))
        return fail(BSSM_ERR_WORKSPACE, "rms_norm backward: workspace too small");
    const void *al[] = {x, weight, grad_out, grad_x, workspace};
    for (const void *p : al)
        if (reinterpret_cast<uintptr_t>(p) & 15)
            return fail(BSSM_ERR_ALIGNMENT, "rms_norm backward: tensors must be 16-byte aligned");
    const int ctas = norm_wave_w(width, dtype, kNormCtas);
    launch_norm_w(width, x, dtype, weight, grad_out, grad_x, rows, eps, workspace, ctas, st);
    if (int rc = check_launch("rms_norm backward")) return rc;
    const long per = (ctas + kRowGroups - 1) / kRowGroups;
    const int groups = static_cast<int>((ctas + per - 1) / per);
    float *const sums = workspace + static_cast<long>(ctas) * width;
    reduce_row_groups_kernel<<<dim3((width + kThreads - 1) / kThreads, groups), kThreads, 0, st>>>(
        workspace, ctas, width, width, per, sums);
    if (int rc = check_launch("rms_norm reduction")) return rc;
    reduce_rows_kernel<<<(width + kThreads - 1) / kThreads, kThreads, 0, st>>>(sums, groups, width, width, grad_weight,
                                                                               width, nullptr);
    return check_launch("rms_norm reduction");
}

long bssm_envelope_epilogue_partial_floats(long batch, long tokens, int heads, int head_dim) {
    // at least one row per CTA of either kernel form
    const long rows = batch * tokens * heads;
    const long rowwise = (rows + kThreads - 1) / kThreads;
    const long tiles = head_dim == 8 || head_dim == 16 ? epi_tiles(batch, tokens, heads, head_dim) : 0;
    return (rowwise > tiles ? rowwise : tiles) * head_dim;
}

int bssm_envelope_epilogue(const void *read, int read_dtype, const void *gate, int gate_dtype, long gate_row_stride,
                           const float *norm_weight, float eps, long batch, long tokens, int heads, int head_dim,
                           void *out, void *stream) {
    if (int rc = epi_check(batch, tokens, heads, head_dim, read_dtype, gate_dtype, gate_row_stride)) return rc;
    if (batch == 0 || tokens == 0) {
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!read || !gate || !norm_weight || !out) return fail(BSSM_ERR_INVALID, "envelope epilogue: null pointer");
    const void *al[] = {read, gate, out};
    for (const void *p : al)
        if (reinterpret_cast<uintptr_t>(p) & 15)
            return fail(BSSM_ERR_ALIGNMENT, "envelope epilogue: tensors must be 16-byte aligned");
    EpiArgs a{read, gate, gate_row_stride, norm_weight, eps, batch, tokens, heads, out, nullptr, nullptr, 0, nullptr};
    launch_epi_hd(a, head_dim, read_dtype, gate_dtype, false, static_cast<cudaStream_t>(stream));
    return check_launch("envelope epilogue");
}

int bssm_envelope_epilogue_backward(const void *read, int read_dtype, const void *gate, int gate_dtype,
                                    long gate_row_stride, const float *norm_weight, float eps, long batch, long tokens,
                                    int heads, int head_dim, const void *grad_out, void *grad_read, void *grad_gate,
                                    long grad_gate_row_stride, float *grad_norm_weight, float *workspace,
                                    long workspace_floats, void *stream) {
    if (int rc = epi_check(batch, tokens, heads, head_dim, read_dtype, gate_dtype, gate_row_stride)) return rc;
    if (grad_gate_row_stride < static_cast<long>(heads) * head_dim || grad_gate_row_stride % 8)
        return fail(BSSM_ERR_INVALID, "envelope epilogue backward: bad gate gradient row stride %ld",
                    grad_gate_row_stride);
    if (!grad_norm_weight) return fail(BSSM_ERR_INVALID, "envelope epilogue backward: null weight gradient");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (batch == 0 || tokens == 0) {
        const cudaError_t err = cudaMemsetAsync(grad_norm_weight, 0, sizeof(float) * head_dim, st);
        if (err != cudaSuccess) return fail(BSSM_ERR_CUDA, "envelope epilogue backward: %s", cudaGetErrorString(err));
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!read || !gate || !norm_weight || !grad_out || !grad_read || !grad_gate || !workspace)
        return fail(BSSM_ERR_INVALID, "envelope epilogue backward: null pointer");
    const long need = bssm_envelope_epilogue_partial_floats(batch, tokens, heads, head_dim);
    if (workspace_floats < need)
        return fail(BSSM_ERR_WORKSPACE, "envelope epilogue backward: workspace of %ld floats, need %ld",
                    workspace_floats, need);
    const void *al[] = {read, gate, grad_out, grad_read, grad_gate};
    for (const void *p : al)
        if (reinterpret_cast<uintptr_t>(p) & 15)
            return fail(BSSM_ERR_ALIGNMENT, "envelope epilogue backward: tensors must be 16-byte aligned");
    EpiArgs a{read, gate, gate_row_stride, norm_weight, eps, batch, tokens, heads, const_cast<void *>(grad_out),
              grad_read, grad_gate, grad_gate_row_stride, workspace};
    launch_epi_hd(a, head_dim, read_dtype, gate_dtype, true, st);
    if (int rc = check_launch("envelope epilogue backward")) return rc;
    const long ctas = epi_ctas(batch, tokens, heads, head_dim);
    reduce_cols_kernel<<<head_dim, kThreads, 0, st>>>(workspace, ctas, head_dim, grad_norm_weight);
    return check_launch("envelope epilogue reduction");
}

}  // extern "C"
