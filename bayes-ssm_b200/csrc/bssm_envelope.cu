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
// Work split: a thread owns two adjacent channels of one batch row and walks
// a span of tokens, keeping the convolution window in registers, so every
// input element is read once (plus a 3-token halo per span).  The channels of
// one head sit in D/2 consecutive lanes, which reduce the head's squared norm
// with xor shuffles.  Streams and heads start at multiples of D/2 channel
// pairs, so a shuffle group never mixes a q/k head with other channels.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "bayes_ssm_b200.h"
#include "bssm_internal.h"

namespace bssm {
namespace env {

constexpr int kThreads = 256;
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

template <bool BF>
__device__ __forceinline__ float2 ld2(const void *base, long idx) {
    if constexpr (BF) {
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162 *>(static_cast<const __nv_bfloat16 *>(base) + idx);
        return __bfloat1622float2(v);
    } else {
        return *reinterpret_cast<const float2 *>(static_cast<const float *>(base) + idx);
    }
}
template <bool BF>
__device__ __forceinline__ void st2(void *base, long idx, float2 v) {
    if constexpr (BF) {
        *reinterpret_cast<__nv_bfloat162 *>(static_cast<__nv_bfloat16 *>(base) + idx) = __float22bfloat162_rn(v);
    } else {
        *reinterpret_cast<float2 *>(static_cast<float *>(base) + idx) = v;
    }
}

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
// torch.nn.functional.softplus with beta 1, threshold 20
__device__ __forceinline__ float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float softplus_grad(float x) { return x > 20.f ? 1.f : sigmoid(x); }

// Sum over the D/2 lanes of this lane's head group (all lanes call it).
__device__ __forceinline__ float head_sum(float v, int group) {
    for (int off = 1; off < group; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

struct ProArgs {
    const void *x;
    const float *w;     // [C][4]
    const float *bias;  // [SW + 2H] or null
    void *k, *q, *v;    // [B*H, T, D] / [B*H, T, HD]
    float *decay;       // [B*H, T, D]
    float *process, *observation;  // [B*H, T]
};

template <bool IN_BF, bool OUT_BF>
__global__ void __launch_bounds__(kThreads) prologue_kernel(const Shape s, const ProArgs a) {
    const int pair = static_cast<int>(blockIdx.x) * kThreads + threadIdx.x;
    const long bb = blockIdx.z;
    const long span = (s.t + s.tsplit - 1) / s.tsplit;
    const long t0 = static_cast<long>(blockIdx.y) * span;
    const long t1 = t0 + span < s.t ? t0 + span : s.t;
    const Chan ch = pair < s.pairs() ? classify(s, pair) : Chan{kIdle, 0, 0};
    const int group = s.d / 2;
    const int c0 = 2 * pair;
    const void *xrow = a.x;
    const long row0 = bb * s.t;
    const long chain = bb * s.heads + ch.head;
    const bool conv = ch.kind <= kV;
    float2 w0{0.f, 0.f}, w1 = w0, w2 = w0, w3 = w0, bias = w0;
    if (conv) {
        w0 = make_float2(a.w[c0 * 4 + 0], a.w[c0 * 4 + 4]);
        w1 = make_float2(a.w[c0 * 4 + 1], a.w[c0 * 4 + 5]);
        w2 = make_float2(a.w[c0 * 4 + 2], a.w[c0 * 4 + 6]);
        w3 = make_float2(a.w[c0 * 4 + 3], a.w[c0 * 4 + 7]);
    } else if ((ch.kind == kDecay || ch.kind == kNoise) && a.bias != nullptr) {
        const int ac = c0 - s.conv_channels();
        bias = make_float2(a.bias[ac], a.bias[ac + 1]);
    }
    // the window x[t-3], x[t-2], x[t-1]
    float2 xm3{0.f, 0.f}, xm2 = xm3, xm1 = xm3;
    if (conv) {
        if (t0 - 3 >= 0) xm3 = ld2<IN_BF>(xrow, (row0 + t0 - 3) * s.in_stride + c0);
        if (t0 - 2 >= 0) xm2 = ld2<IN_BF>(xrow, (row0 + t0 - 2) * s.in_stride + c0);
        if (t0 - 1 >= 0) xm1 = ld2<IN_BF>(xrow, (row0 + t0 - 1) * s.in_stride + c0);
    }
#pragma unroll 4
    for (long t = t0; t < t1; ++t) {
        float2 x{0.f, 0.f};
        if (ch.kind != kIdle) x = ld2<IN_BF>(xrow, (row0 + t) * s.in_stride + c0);
        float2 o{0.f, 0.f};
        float ss = 0.f;
        if (conv) {
            const float cx = fmaf(w3.x, x.x, fmaf(w2.x, xm1.x, fmaf(w1.x, xm2.x, w0.x * xm3.x)));
            const float cy = fmaf(w3.y, x.y, fmaf(w2.y, xm1.y, fmaf(w1.y, xm2.y, w0.y * xm3.y)));
            o = make_float2(cx * sigmoid(cx), cy * sigmoid(cy));
            ss = ch.kind == kV ? 0.f : o.x * o.x + o.y * o.y;
            xm3 = xm2;
            xm2 = xm1;
            xm1 = x;
        }
        ss = head_sum(ss, group);  // q and k heads only; other groups sum zeros
        if (ch.kind == kQ || ch.kind == kK) {
            const float r = 1.0f / fmaxf(sqrtf(ss), kNormEps);
            o.x *= r;
            o.y *= r;
            st2<OUT_BF>(ch.kind == kQ ? a.q : a.k, (chain * s.t + t) * s.d + ch.within, o);
        } else if (ch.kind == kV) {
            st2<OUT_BF>(a.v, (chain * s.t + t) * s.hd + ch.within, o);
        } else if (ch.kind == kDecay) {
            const float2 dcy = make_float2(expf(-softplus(x.x + bias.x)), expf(-softplus(x.y + bias.y)));
            *reinterpret_cast<float2 *>(a.decay + (chain * s.t + t) * s.d + ch.within) = dcy;
        } else if (ch.kind == kNoise) {
            a.process[chain * s.t + t] = softplus(x.x + bias.x) + kNoiseFloor;
            a.observation[chain * s.t + t] = softplus(x.y + bias.y) + kNoiseFloor;
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
    float *partial;  // [B * tsplit][4 C + SW + 2H]
};

// Backward of one token span: walk the tokens downwards, recompute the
// forward at each, and keep the last four convolution-input gradients so that
// gx[t] = sum_j w_j gc[t + 3 - j].  The span also recomputes the 3 tokens
// after it (their gc feeds its last gx) without counting them in the weight
// gradient, which their own span does.
template <bool IN_BF, bool OUT_BF>
__global__ void __launch_bounds__(kThreads) prologue_backward_kernel(const Shape s, const EnvBwdArgs a) {
    const int pair = static_cast<int>(blockIdx.x) * kThreads + threadIdx.x;
    const long bb = blockIdx.z;
    const long span = (s.t + s.tsplit - 1) / s.tsplit;
    const long t0 = static_cast<long>(blockIdx.y) * span;
    const long t1 = t0 + span < s.t ? t0 + span : s.t;
    const long hi = t1 + 3 < s.t ? t1 + 3 : s.t;
    const Chan ch = pair < s.pairs() ? classify(s, pair) : Chan{kIdle, 0, 0};
    const int group = s.d / 2;
    const int c0 = 2 * pair;
    const long row0 = bb * s.t;
    const long chain = bb * s.heads + ch.head;
    const bool conv = ch.kind <= kV;
    const int C = s.conv_channels();
    float *const part = a.partial + (bb * s.tsplit + blockIdx.y) * static_cast<long>(s.partial_cols());
    float2 w0{0.f, 0.f}, w1 = w0, w2 = w0, w3 = w0, bias = w0;
    if (conv) {
        w0 = make_float2(a.w[c0 * 4 + 0], a.w[c0 * 4 + 4]);
        w1 = make_float2(a.w[c0 * 4 + 1], a.w[c0 * 4 + 5]);
        w2 = make_float2(a.w[c0 * 4 + 2], a.w[c0 * 4 + 6]);
        w3 = make_float2(a.w[c0 * 4 + 3], a.w[c0 * 4 + 7]);
    } else if ((ch.kind == kDecay || ch.kind == kNoise) && a.bias != nullptr) {
        const int ac = c0 - C;
        bias = make_float2(a.bias[ac], a.bias[ac + 1]);
    }
    auto ldx = [&](long t) -> float2 {
        return (t >= 0 && ch.kind != kIdle) ? ld2<IN_BF>(a.x, (row0 + t) * s.in_stride + c0) : make_float2(0.f, 0.f);
    };
    // x[t-3 .. t] for t = hi - 1 (conv channels only)
    float2 x3{0.f, 0.f}, x2 = x3, x1 = x3, x0 = x3;  // x0 = x[t], x1 = x[t-1], ...
    if (conv && hi > t0) {
        x0 = ldx(hi - 1);
        x1 = ldx(hi - 2);
        x2 = ldx(hi - 3);
    }
    float2 gp1{0.f, 0.f}, gp2 = gp1, gp3 = gp1;  // gc[t+1], gc[t+2], gc[t+3]
    float2 gw0{0.f, 0.f}, gw1 = gw0, gw2 = gw0, gw3 = gw0, gb = gw0;
#pragma unroll 2
    for (long t = hi - 1; t >= t0; --t) {
        float2 gc{0.f, 0.f};
        float ss = 0.f, dot = 0.f;
        float2 o{0.f, 0.f}, g{0.f, 0.f}, ds{0.f, 0.f};
        if (conv) {
            x3 = ldx(t - 3);
            const float cx = fmaf(w3.x, x0.x, fmaf(w2.x, x1.x, fmaf(w1.x, x2.x, w0.x * x3.x)));
            const float cy = fmaf(w3.y, x0.y, fmaf(w2.y, x1.y, fmaf(w1.y, x2.y, w0.y * x3.y)));
            const float sx = sigmoid(cx), sy = sigmoid(cy);
            o = make_float2(cx * sx, cy * sy);
            ds = make_float2(sx * fmaf(cx, 1.f - sx, 1.f), sy * fmaf(cy, 1.f - sy, 1.f));  // silu'
            const void *gsrc = ch.kind == kQ ? a.gq : ch.kind == kK ? a.gk : a.gv;
            if (gsrc != nullptr)
                g = ld2<OUT_BF>(gsrc, (chain * s.t + t) * (ch.kind == kV ? s.hd : s.d) + ch.within);
            if (ch.kind != kV) ss = o.x * o.x + o.y * o.y;
        }
        ss = head_sum(ss, group);
        if (ch.kind == kQ || ch.kind == kK) {
            const float n = sqrtf(ss);
            const float r = 1.0f / fmaxf(n, kNormEps);
            o.x *= r;  // the normalised output y
            o.y *= r;
            dot = o.x * g.x + o.y * g.y;
        }
        dot = head_sum(dot, group);
        if (ch.kind == kQ || ch.kind == kK) {
            // y = s / max(|s|, eps): dy/ds = (I - y y^T) / |s| above eps, I / eps below
            const float n = sqrtf(ss), r = 1.0f / fmaxf(n, kNormEps);
            const float dd = n > kNormEps ? dot : 0.f;
            gc = make_float2((g.x - o.x * dd) * r * ds.x, (g.y - o.y * dd) * r * ds.y);
        } else if (ch.kind == kV) {
            gc = make_float2(g.x * ds.x, g.y * ds.y);
        }
        if (t < t1) {
            if (conv) {
                const float2 gx = make_float2(fmaf(w0.x, gp3.x, fmaf(w1.x, gp2.x, fmaf(w2.x, gp1.x, w3.x * gc.x))),
                                              fmaf(w0.y, gp3.y, fmaf(w1.y, gp2.y, fmaf(w2.y, gp1.y, w3.y * gc.y))));
                st2<IN_BF>(a.gx, (row0 + t) * a.gx_stride + c0, gx);
                gw0 = make_float2(fmaf(gc.x, x3.x, gw0.x), fmaf(gc.y, x3.y, gw0.y));
                gw1 = make_float2(fmaf(gc.x, x2.x, gw1.x), fmaf(gc.y, x2.y, gw1.y));
                gw2 = make_float2(fmaf(gc.x, x1.x, gw2.x), fmaf(gc.y, x1.y, gw2.y));
                gw3 = make_float2(fmaf(gc.x, x0.x, gw3.x), fmaf(gc.y, x0.y, gw3.y));
            } else if (ch.kind == kDecay) {
                const float2 xv = ldx(t);
                const float2 gd = a.gdecay != nullptr
                                      ? *reinterpret_cast<const float2 *>(a.gdecay + (chain * s.t + t) * s.d + ch.within)
                                      : make_float2(0.f, 0.f);
                const float zx = xv.x + bias.x, zy = xv.y + bias.y;
                // d/dz exp(-softplus(z)) = -exp(-softplus(z)) softplus'(z)
                const float2 gz = make_float2(-gd.x * expf(-softplus(zx)) * softplus_grad(zx),
                                              -gd.y * expf(-softplus(zy)) * softplus_grad(zy));
                st2<IN_BF>(a.gx, (row0 + t) * a.gx_stride + c0, gz);
                gb = make_float2(gb.x + gz.x, gb.y + gz.y);
            } else if (ch.kind == kNoise) {
                const float2 xv = ldx(t);
                const float gpv = a.gprocess != nullptr ? a.gprocess[chain * s.t + t] : 0.f;
                const float gov = a.gobservation != nullptr ? a.gobservation[chain * s.t + t] : 0.f;
                const float2 gz = make_float2(gpv * softplus_grad(xv.x + bias.x), gov * softplus_grad(xv.y + bias.y));
                st2<IN_BF>(a.gx, (row0 + t) * a.gx_stride + c0, gz);
                gb = make_float2(gb.x + gz.x, gb.y + gz.y);
            }
        }
        gp3 = gp2;
        gp2 = gp1;
        gp1 = gc;
        x0 = x1;
        x1 = x2;
        x2 = x3;
    }
    if (conv) {
        float4 *pw = reinterpret_cast<float4 *>(part + c0 * 4);  // [c][4], c0 even: 32-byte aligned
        pw[0] = make_float4(gw0.x, gw1.x, gw2.x, gw3.x);
        pw[1] = make_float4(gw0.y, gw1.y, gw2.y, gw3.y);
    } else if (ch.kind == kDecay || ch.kind == kNoise) {
        const int ac = c0 - C;
        part[4 * C + ac] = gb.x;
        part[4 * C + ac + 1] = gb.y;
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

int pick_tsplit(long b, long t) {
    // enough CTAs for every SM several times over, spans of at least 32 tokens
    int ts = 1;
    while (b * ts < 4 * 148 && t / (2 * ts) >= 32) ts *= 2;
    return ts;
}

}  // namespace env
}  // namespace bssm

using namespace bssm;
using namespace bssm::env;

extern "C" {

long bssm_envelope_partial_floats(long batch, long tokens, int heads, int key_dim, int head_dim) {
    Shape s{batch, tokens, heads, key_dim, head_dim, 0, 1};
    return batch * pick_tsplit(batch, tokens) * static_cast<long>(s.partial_cols());
}

int bssm_envelope_prologue(const void *projected, int in_dtype, long batch, long tokens, int heads, int key_dim,
                           int head_dim, long row_stride, const float *conv_weight, const float *aux_bias,
                           void *keys, void *queries, void *values, int out_dtype, float *decay, float *process,
                           float *observation, void *stream) {
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
    s.tsplit = pick_tsplit(batch, tokens);
    const ProArgs a{projected, conv_weight, aux_bias, keys, queries, values, decay, process, observation};
    const dim3 grid((s.pairs() + kThreads - 1) / kThreads, s.tsplit, static_cast<unsigned>(batch));
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (in_dtype == BSSM_BF16) {
        if (out_dtype == BSSM_BF16) prologue_kernel<true, true><<<grid, kThreads, 0, st>>>(s, a);
        else prologue_kernel<true, false><<<grid, kThreads, 0, st>>>(s, a);
    } else {
        if (out_dtype == BSSM_BF16) prologue_kernel<false, true><<<grid, kThreads, 0, st>>>(s, a);
        else prologue_kernel<false, false><<<grid, kThreads, 0, st>>>(s, a);
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
    s.tsplit = pick_tsplit(batch, tokens);
    const long need = batch * s.tsplit * static_cast<long>(pcols);
    if (workspace_floats < need)
        return fail(BSSM_ERR_WORKSPACE, "envelope backward: workspace of %ld floats, need %ld", workspace_floats, need);
    if (reinterpret_cast<uintptr_t>(workspace) & 31)
        return fail(BSSM_ERR_ALIGNMENT, "envelope backward: workspace must be 32-byte aligned");
    const void *aligned8[] = {projected, grad_projected, grad_keys, grad_queries, grad_values, grad_decay};
    for (const void *p : aligned8)
        if (reinterpret_cast<uintptr_t>(p) & 7)
            return fail(BSSM_ERR_ALIGNMENT, "envelope backward: tensors must be 8-byte aligned");
    const EnvBwdArgs a{projected, conv_weight, aux_bias, grad_keys, grad_queries, grad_values, grad_decay, grad_process,
                    grad_observation, grad_projected, grad_row_stride, workspace};
    const dim3 grid((s.pairs() + kThreads - 1) / kThreads, s.tsplit, static_cast<unsigned>(batch));
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (in_dtype == BSSM_BF16) {
        if (out_dtype == BSSM_BF16) prologue_backward_kernel<true, true><<<grid, kThreads, 0, st>>>(s, a);
        else prologue_backward_kernel<true, false><<<grid, kThreads, 0, st>>>(s, a);
    } else {
        if (out_dtype == BSSM_BF16) prologue_backward_kernel<false, true><<<grid, kThreads, 0, st>>>(s, a);
        else prologue_backward_kernel<false, false><<<grid, kThreads, 0, st>>>(s, a);
    }
    if (int rc = check_launch("envelope prologue backward")) return rc;
    reduce_rows_kernel<<<(cols + kThreads - 1) / kThreads, kThreads, 0, st>>>(workspace, batch * s.tsplit, cols, pcols,
                                                                               grad_conv_weight, 4 * C, grad_aux_bias);
    return check_launch("envelope reduction");
}

}  // extern "C"
