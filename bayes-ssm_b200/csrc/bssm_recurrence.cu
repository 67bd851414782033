// bssm_recurrence.cu -- chunked forward and chunk-replay backward of the
// dense-covariance Bayesian layer with diagonal dynamics, for sm_100a.
//
// Recurrence per token (A = diag(a), state M [D,M], P [D,D]):
//   Pbar = A P A + p I, u = Pbar k, s = r + k.u, beta = 1/max(s, floor),
//   e = v - (A M)^T k, M' = A M + beta u e^T, P' = Pbar - beta u u^T,
//   y = M'^T q.
// (catid/bayes-ssm bayes_ssm/bayesian_layer.py:153-181 and :207-251; the
// fixed-dynamics constants of :360-400.)
//
// Work decomposition.  A chain is served by LPC = D lanes: lane i owns row i
// of P (and of the covariance adjoint R) and M/D columns of the mean (and of
// its adjoint).  With that split the predict/update is lane-local except for
// one gather of u (D shuffles); the readout y_c = sum_i M_ic q_i is lane-local.
// The adjoint needs four reduce-scatters of D-vectors (gq, gM'e, M ge, the
// decay gradient of the mean) and one gather of the gain adjoint.
//
// Backward (one launch for the whole sequence): each chain walks its chunks
// from last to first.  Inside chunk c it replays the chunk from the saved
// boundary state, storing the state every S tokens into a global workspace
// (phase A), then for each S-token sub-chunk from last to first replays the
// sub-chunk into shared-memory history and runs the reverse step over it
// (phase B).  No per-token history ever reaches global memory and there is
// no per-chunk launch.
#include <cuda.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "bayes_ssm_b200.h"
#include "bssm_common.cuh"
#include "bssm_internal.h"

namespace bssm {

// Threads per CTA for a key dimension (chains per CTA = threads / D).
template <int D>
struct Launch {
    static constexpr int kThreads = (D >= 4) ? 128 : 64;
    static constexpr int kChains = kThreads / D;
};

// Sub-chunk length (tokens of shared-memory history per chain).
template <int D>
struct SubChunk {
    static constexpr int S = 4;
};

// Floats of phase-A workspace per lane per saved state: the lane's M mean
// entries and its covariance row, padded to a 16-byte multiple.
template <int D, int M>
struct Slot {
    static constexpr int kLane = ((M + D) + 3) / 4 * 4;
    static constexpr int kChain = kLane * D;
};

// Per-token inputs of one lane.
template <int D, int M>
struct Token {
    static constexpr int CPL = M / D;
    float k[D], a[D], q[D], v[CPL], gy[CPL];
    float p, r;
};

template <int D, int M, bool FIXED, bool WANT_Q, bool WANT_GY, typename TIn>
__device__ __forceinline__ void load_token(Token<D, M> &tk, const TIn *keys, const TIn *values,
                                           const TIn *queries, const float *decay,
                                           const float *process, const float *observation,
                                           const float *gy, long row, int col0) {
    constexpr int CPL = M / D;
    load_vec<D>(keys + row * D, tk.k);
    load_vec<CPL>(values + row * M + col0, tk.v);
    if constexpr (WANT_Q) load_vec<D>(queries + row * D, tk.q);
    if constexpr (FIXED) {
#pragma unroll
        for (int j = 0; j < D; ++j) tk.a[j] = kFixedDecay;
        tk.p = kFixedProcess;
        tk.r = kFixedObservation;
    } else {
        load_vec<D>(decay + row * D, tk.a);
        tk.p = __ldg(process + row);
        tk.r = __ldg(observation + row);
    }
    if constexpr (WANT_GY) {
        if (gy != nullptr) {
            load_vec<CPL>(gy + row * M + col0, tk.gy);
        } else {
#pragma unroll
            for (int l = 0; l < CPL; ++l) tk.gy[l] = 0.f;
        }
    }
}

// Quantities of one forward step the backward stores as history.
template <int D, int M>
struct StepInfo {
    float u[D];
    float e[M / D];
    float u_own, beta, s;
};

// One predict/update step on the lane's state slice (in place).
template <int D, int M>
__device__ __forceinline__ void forward_step(const LaneGroup<D> &g, const Token<D, M> &tk,
                                             float (&Mc)[M / D][D], float (&P)[D], float floor_,
                                             StepInfo<D, M> &si) {
    constexpr int CPL = M / D;
    const int own = g.sub;
    float wk[D];
#pragma unroll
    for (int j = 0; j < D; ++j) wk[j] = tk.a[j] * tk.k[j];
    const float k_own = pick(tk.k, own);
    const float a_own = pick(tk.a, own);
    // u_own = a_own * sum_j P_own,j a_j k_j + p k_own
    float z = 0.f;
#pragma unroll
    for (int j = 0; j < D; ++j) z = fmaf(P[j], wk[j], z);
    const float u_own = fmaf(a_own, z, tk.p * k_own);
    // innovation e_c = v_c - sum_i a_i M_ic k_i (independent of u)
#pragma unroll
    for (int l = 0; l < CPL; ++l) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < D; ++i) acc = fmaf(Mc[l][i], wk[i], acc);
        si.e[l] = tk.v[l] - acc;
    }
    g.gather(u_own, si.u);
    float s = tk.r;
#pragma unroll
    for (int j = 0; j < D; ++j) s = fmaf(tk.k[j], si.u[j], s);
    // clamp_min semantics: a NaN s stays NaN
    const float beta = 1.0f / (s < floor_ ? floor_ : s);
#pragma unroll
    for (int l = 0; l < CPL; ++l) {
        const float be = beta * si.e[l];
#pragma unroll
        for (int i = 0; i < D; ++i) Mc[l][i] = fmaf(tk.a[i], Mc[l][i], be * si.u[i]);
    }
    // Row own of P' = A P A + p I - beta u u^T.  Every product is formed
    // from commutative pairs (a_i a_j, u_i u_j), so lane i and lane j compute
    // bit-identical P'_ij and P'_ji: the covariance stays exactly symmetric.
#pragma unroll
    for (int j = 0; j < D; ++j) {
        const float upd = fmaf(-beta, u_own * si.u[j], (a_own * tk.a[j]) * P[j]);
        P[j] = (j == own) ? upd + tk.p : upd;
    }
    si.u_own = u_own;
    si.beta = beta;
    si.s = s;
}

template <int D, int M>
__device__ __forceinline__ void readout(const Token<D, M> &tk, const float (&Mc)[M / D][D],
                                        float (&y)[M / D]) {
#pragma unroll
    for (int l = 0; l < M / D; ++l) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < D; ++i) acc = fmaf(Mc[l][i], tk.q[i], acc);
        y[l] = acc;
    }
}

// Lane's slice of a [D,M] mean at `base`: columns col0 .. col0+CPL-1.
template <int D, int M>
__device__ __forceinline__ void load_mean_cols(const float *base, int col0, float (&Mc)[M / D][D]) {
    constexpr int CPL = M / D;
#pragma unroll
    for (int i = 0; i < D; ++i) {
        float row[CPL];
        load_vec<CPL>(base + i * M + col0, row);
#pragma unroll
        for (int l = 0; l < CPL; ++l) Mc[l][i] = row[l];
    }
}

template <int D, int M>
__device__ __forceinline__ void store_mean_cols(float *base, int col0, const float (&Mc)[M / D][D]) {
    constexpr int CPL = M / D;
#pragma unroll
    for (int i = 0; i < D; ++i) {
        float row[CPL];
#pragma unroll
        for (int l = 0; l < CPL; ++l) row[l] = Mc[l][i];
        store_vec<CPL>(base + i * M + col0, row);
    }
}

// ===========================================================================
// Forward
// ===========================================================================
template <int D, int M, bool FIXED, typename TIn>
__global__ void __launch_bounds__(Launch<D>::kThreads)
    forward_kernel(const FwdArgs<TIn> A) {
    constexpr int CPL = M / D;
    const LaneGroup<D> g;
    const long chain = (static_cast<long>(blockIdx.x) * Launch<D>::kThreads + threadIdx.x) / D;
    if (chain >= A.n) return;  // whole lane groups retire together
    const int own = g.sub;
    const int col0 = own * CPL;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;

    float Mc[CPL][D], P[D];
    if (A.mean0 != nullptr) {
        load_mean_cols<D, M>(A.mean0 + chain * D * M, col0, Mc);
    } else {
#pragma unroll
        for (int l = 0; l < CPL; ++l)
#pragma unroll
            for (int i = 0; i < D; ++i) Mc[l][i] = 0.f;
    }
    if (A.cov0 != nullptr) {
        const float *c0 = A.cov0 + chain * D * D;
#pragma unroll
        for (int j = 0; j < D; ++j) P[j] = 0.5f * (c0[own * D + j] + c0[j * D + own]);
    } else {
#pragma unroll
        for (int j = 0; j < D; ++j) P[j] = (j == own) ? 1.f : 0.f;
    }

    float *bm = A.bmean + chain * (nb + 1) * D * M;
    float *bc = A.bcov + chain * (nb + 1) * D * D;
    Token<D, M> cur, nxt;
    if (T > 0)
        load_token<D, M, FIXED, true, false>(cur, A.keys, A.values, A.queries, A.decay, A.process,
                                             A.observation, nullptr, chain * T, col0);
    int in_chunk = 0;
    long c = 0;
    const long rs_slots = replay_slots_per_chunk(T, L);
    for (long ti = 0; ti < T; ++ti) {
        if (in_chunk == 0) {
            store_mean_cols<D, M>(bm + c * D * M, col0, Mc);
            store_vec<D>(bc + c * D * D + own * D, P);
            ++c;
        } else if (A.rs != nullptr && in_chunk % kReplaySpan == 0) {
            const long base = replay_state_base(chain, nb, rs_slots, c - 1, in_chunk / kReplaySpan,
                                                replay_state_floats(D, M));
            rs_put_mean_cols<D, M, CPL>(A.rs, base, col0, Mc);
            rs_put_row<D, M>(A.rs, base, own, P);
        }
        if (++in_chunk == L) in_chunk = 0;
        const long row = chain * T + ti;
        if (ti + 1 < T)
            load_token<D, M, FIXED, true, false>(nxt, A.keys, A.values, A.queries, A.decay,
                                                 A.process, A.observation, nullptr, row + 1, col0);
        StepInfo<D, M> si;
        forward_step<D, M>(g, cur, Mc, P, A.floor, si);
        if (A.rs != nullptr) {
            replay_gains(A.rs, A.n, T, L, D, M)[row * D + own] = si.u_own;
            if (own == 0) replay_gain_scales(A.rs, A.n, T, L, D, M)[row] = signed_gain_scale(si.beta, si.s, A.floor);
        }
        float y[CPL];
        readout<D, M>(cur, Mc, y);
        store_vec<CPL>(A.out + row * M + col0, y);
        cur = nxt;
    }
    store_mean_cols<D, M>(bm + nb * D * M, col0, Mc);
    store_vec<D>(bc + nb * D * D + own * D, P);
    store_mean_cols<D, M>(A.mean_final + chain * D * M, col0, Mc);
    store_vec<D>(A.cov_final + chain * D * D + own * D, P);
}

// ===========================================================================
// Backward
// ===========================================================================

// Shared-memory history of one chain for one S-token sub-chunk.  Every
// lane-private block is interleaved in 4-float chunks across the group's
// lanes so that the 128-bit accesses of a group hit distinct banks.
template <int D, int M, int S>
struct History {
    static constexpr int LPC = D;
    static constexpr int kMean = M;              // floats of mean per lane per token
    static constexpr int kRow = D;               // floats of covariance row per lane per token
    static constexpr int oM = 0;                 // [S][M*D]
    static constexpr int oP = oM + S * M * D;    // [S][D*D]
    static constexpr int oU = oP + S * D * D;    // [S][D]
    static constexpr int oK = oU + S * D;        // [S][D]
    static constexpr int oA = oK + S * D;        // [S][D]
    static constexpr int oQ = oA + S * D;        // [S][D]
    static constexpr int oE = oQ + S * D;        // [S][M]
    static constexpr int oG = oE + S * M;        // [S][M]
    static constexpr int oB = oG + S * M;        // [S][4]: beta, s, p, -
    static constexpr int kFloats = oB + S * 4;

    // Offset of the 4-float chunk x of lane `sub`'s block of `block` floats.
    template <int BLOCK>
    __device__ static __forceinline__ int chunk_off(int x, int sub) {
        if constexpr (BLOCK >= 4) {
            return x * (LPC * 4) + sub * 4;
        } else {
            return sub * BLOCK;
        }
    }
    template <int BLOCK>
    __device__ static __forceinline__ void put(float *base, int sub, const float (&v)[BLOCK]) {
        if constexpr (BLOCK >= 4) {
#pragma unroll
            for (int x = 0; x < BLOCK / 4; ++x)
                *reinterpret_cast<float4 *>(base + chunk_off<BLOCK>(x, sub)) =
                    make_float4(v[4 * x], v[4 * x + 1], v[4 * x + 2], v[4 * x + 3]);
        } else if constexpr (BLOCK == 2) {
            *reinterpret_cast<float2 *>(base + sub * 2) = make_float2(v[0], v[1]);
        } else {
            base[sub] = v[0];
        }
    }
    template <int BLOCK>
    __device__ static __forceinline__ void get(const float *base, int sub, float (&v)[BLOCK]) {
        if constexpr (BLOCK >= 4) {
#pragma unroll
            for (int x = 0; x < BLOCK / 4; ++x) {
                const float4 w = *reinterpret_cast<const float4 *>(base + chunk_off<BLOCK>(x, sub));
                v[4 * x] = w.x; v[4 * x + 1] = w.y; v[4 * x + 2] = w.z; v[4 * x + 3] = w.w;
            }
        } else if constexpr (BLOCK == 2) {
            const float2 w = *reinterpret_cast<const float2 *>(base + sub * 2);
            v[0] = w.x; v[1] = w.y;
        } else {
            v[0] = base[sub];
        }
    }
    // all D floats of a shared per-token vector
    __device__ static __forceinline__ void get_all(const float *base, float (&v)[D]) {
        if constexpr (D >= 4) {
#pragma unroll
            for (int x = 0; x < D; x += 4) {
                const float4 w = *reinterpret_cast<const float4 *>(base + x);
                v[x] = w.x; v[x + 1] = w.y; v[x + 2] = w.z; v[x + 3] = w.w;
            }
        } else if constexpr (D == 2) {
            const float2 w = *reinterpret_cast<const float2 *>(base);
            v[0] = w.x; v[1] = w.y;
        } else {
            v[0] = base[0];
        }
    }
};

template <int D, int M>
__device__ __forceinline__ void flatten_mean(const float (&Mc)[M / D][D], float (&flat)[M]) {
#pragma unroll
    for (int l = 0; l < M / D; ++l)
#pragma unroll
        for (int i = 0; i < D; ++i) flat[l * D + i] = Mc[l][i];
}
template <int D, int M>
__device__ __forceinline__ void unflatten_mean(const float (&flat)[M], float (&Mc)[M / D][D]) {
#pragma unroll
    for (int l = 0; l < M / D; ++l)
#pragma unroll
        for (int i = 0; i < D; ++i) Mc[l][i] = flat[l * D + i];
}

template <int D, int M, int S, bool FIXED, bool NEED_DYN, bool NEED_INIT, typename TIn>
__global__ void __launch_bounds__(Launch<D>::kThreads)
    backward_kernel(const BwdArgs<TIn> A) {
    constexpr int CPL = M / D;
    using H = History<D, M, S>;
    extern __shared__ __align__(16) float smem[];
    const LaneGroup<D> g;
    const int group_in_cta = threadIdx.x / D;
    const long chain = static_cast<long>(blockIdx.x) * Launch<D>::kChains + group_in_cta;
    if (chain >= A.n) return;
    float *hist = smem + group_in_cta * H::kFloats;
    const int own = g.sub;
    const int col0 = own * CPL;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;
    const int nsub_max = (static_cast<int>(L < T ? L : T) + S - 1) / S;
    const float floor_ = A.floor;
    const float *bm = A.bmean + chain * (nb + 1) * D * M;
    const float *bc = A.bcov + chain * (nb + 1) * D * D;
    // phase-A workspace: (nsub_max - 1) saved states per chain
    using SL = Slot<D, M>;
    float *ws = A.ws + chain * static_cast<long>(nsub_max > 1 ? nsub_max - 1 : 0) * SL::kChain;

    // carried adjoints: gM (mean columns) and R = sym(dL/dP) (covariance row)
    float gM[CPL][D], R[D];
    if (A.gmf != nullptr) {
        load_mean_cols<D, M>(A.gmf + chain * D * M, col0, gM);
    } else {
#pragma unroll
        for (int l = 0; l < CPL; ++l)
#pragma unroll
            for (int i = 0; i < D; ++i) gM[l][i] = 0.f;
    }
    if (A.gcf != nullptr) {
        const float *gc = A.gcf + chain * D * D;
#pragma unroll
        for (int j = 0; j < D; ++j) R[j] = 0.5f * (gc[own * D + j] + gc[j * D + own]);
    } else {
#pragma unroll
        for (int j = 0; j < D; ++j) R[j] = 0.f;
    }
    // post-update mean of the token after the current span (M_T initially)
    float Mnext[CPL][D];
    load_mean_cols<D, M>(bm + nb * D * M, col0, Mnext);

    for (long ci = nb - 1; ci >= 0; --ci) {
        const long t0 = ci * L;
        const int len = static_cast<int>((T - t0) < L ? (T - t0) : L);
        const int nsub = (len + S - 1) / S;

        // ---- phase A: states at sub-chunk starts 1 .. nsub-1 -> workspace
        // (skipped when the forward saved them)
        if (nsub > 1 && A.rs == nullptr) {
            float Mc[CPL][D], P[D];
            load_mean_cols<D, M>(bm + ci * D * M, col0, Mc);
            load_vec<D>(bc + ci * D * D + own * D, P);
            const int steps = (nsub - 1) * S;
            Token<D, M> cur, nxt;
            load_token<D, M, FIXED, false, false>(cur, A.keys, A.values, A.queries, A.decay,
                                                  A.process, A.observation, nullptr,
                                                  chain * T + t0, col0);
            for (int x = 0; x < steps; ++x) {
                const long row = chain * T + t0 + x;
                if (x + 1 < steps)
                    load_token<D, M, FIXED, false, false>(nxt, A.keys, A.values, A.queries,
                                                          A.decay, A.process, A.observation,
                                                          nullptr, row + 1, col0);
                StepInfo<D, M> si;
                forward_step<D, M>(g, cur, Mc, P, floor_, si);
                if ((x + 1) % S == 0) {
                    float *slot = ws + static_cast<long>((x + 1) / S - 1) * SL::kChain + own * SL::kLane;
                    float flat[M];
                    flatten_mean<D, M>(Mc, flat);
                    store_vec<M>(slot, flat);
                    store_vec<D>(slot + M, P);
                }
                cur = nxt;
            }
        }

        // ---- phase B: per sub-chunk, replay into history then reverse
        for (int j = nsub - 1; j >= 0; --j) {
            const long s0 = t0 + static_cast<long>(j) * S;
            const int slen = (len - j * S) < S ? (len - j * S) : S;
            float Mc[CPL][D], P[D];
            if (j == 0) {
                load_mean_cols<D, M>(bm + ci * D * M, col0, Mc);
                load_vec<D>(bc + ci * D * D + own * D, P);
            } else if (A.rs != nullptr) {
                const long base = replay_state_base(chain, nb, nsub_max - 1, ci, j, replay_state_floats(D, M));
                rs_get_mean_cols<D, M, CPL>(A.rs, base, col0, Mc);
                rs_get_row<D, M>(A.rs, base, own, P);
            } else {
                const float *slot = ws + static_cast<long>(j - 1) * SL::kChain + own * SL::kLane;
                // written earlier by this kernel: coherent loads, not the read-only path
                float flat[M];
                load_vec_coherent<M>(slot, flat);
                unflatten_mean<D, M>(flat, Mc);
                if constexpr (D % 4 == 0) {
                    load_vec_coherent<D>(slot + M, P);
                } else {
#pragma unroll
                    for (int jj = 0; jj < D; ++jj) P[jj] = slot[M + jj];
                }
            }
            float Mstart[CPL][D];
#pragma unroll
            for (int l = 0; l < CPL; ++l)
#pragma unroll
                for (int i = 0; i < D; ++i) Mstart[l][i] = Mc[l][i];

            g.sync();  // previous reverse pass finished reading the history
            Token<D, M> cur, nxt;
            load_token<D, M, FIXED, true, true>(cur, A.keys, A.values, A.queries, A.decay,
                                                A.process, A.observation, A.gy, chain * T + s0,
                                                col0);
            for (int tau = 0; tau < slen; ++tau) {
                const long row = chain * T + s0 + tau;
                if (tau + 1 < slen)
                    load_token<D, M, FIXED, true, true>(nxt, A.keys, A.values, A.queries, A.decay,
                                                        A.process, A.observation, A.gy, row + 1,
                                                        col0);
                {
                    float flat[M];
                    flatten_mean<D, M>(Mc, flat);
                    H::template put<M>(hist + H::oM + tau * M * D, own, flat);
                    H::template put<D>(hist + H::oP + tau * D * D, own, P);
                }
                StepInfo<D, M> si;
                forward_step<D, M>(g, cur, Mc, P, floor_, si);
                hist[H::oU + tau * D + own] = si.u_own;
                hist[H::oK + tau * D + own] = pick(cur.k, own);
                hist[H::oA + tau * D + own] = pick(cur.a, own);
                hist[H::oQ + tau * D + own] = pick(cur.q, own);
                store_vec<CPL>(hist + H::oE + tau * M + col0, si.e);
                store_vec<CPL>(hist + H::oG + tau * M + col0, cur.gy);
                if (own == 0)
                    *reinterpret_cast<float4 *>(hist + H::oB + tau * 4) =
                        make_float4(si.beta, si.s, cur.p, 0.f);
                cur = nxt;
            }
            g.sync();

            for (int tau = slen - 1; tau >= 0; --tau) {
                const long row = chain * T + s0 + tau;
                float k[D], a[D], q[D], u[D];
                H::get_all(hist + H::oK + tau * D, k);
                H::get_all(hist + H::oA + tau * D, a);
                H::get_all(hist + H::oQ + tau * D, q);
                H::get_all(hist + H::oU + tau * D, u);
                const float k_own = hist[H::oK + tau * D + own];
                const float a_own = hist[H::oA + tau * D + own];
                const float u_own = hist[H::oU + tau * D + own];
                const float4 bsp = *reinterpret_cast<const float4 *>(hist + H::oB + tau * 4);
                const float beta = bsp.x, s = bsp.y, p = bsp.z;
                float e[CPL], gyv[CPL];
#pragma unroll
                for (int l = 0; l < CPL; ++l) {
                    e[l] = hist[H::oE + tau * M + col0 + l];
                    gyv[l] = hist[H::oG + tau * M + col0 + l];
                }
                float Mp[CPL][D], Mn[CPL][D], Pp[D];
                {
                    float flat[M];
                    H::template get<M>(hist + H::oM + tau * M * D, own, flat);
                    unflatten_mean<D, M>(flat, Mp);
                    if (tau + 1 < slen) {
                        H::template get<M>(hist + H::oM + (tau + 1) * M * D, own, flat);
                        unflatten_mean<D, M>(flat, Mn);
                    } else {
#pragma unroll
                        for (int l = 0; l < CPL; ++l)
#pragma unroll
                            for (int i = 0; i < D; ++i) Mn[l][i] = Mnext[l][i];
                    }
                    H::template get<D>(hist + H::oP + tau * D * D, own, Pp);
                }

                // gradient reaching the post-update mean
#pragma unroll
                for (int l = 0; l < CPL; ++l)
#pragma unroll
                    for (int i = 0; i < D; ++i) gM[l][i] = fmaf(q[i], gyv[l], gM[l][i]);

                // partial sums over this lane's columns
                float part[4][D];
                float ge[CPL];
                float gb = 0.f;
#pragma unroll
                for (int l = 0; l < CPL; ++l) {
                    float acc = 0.f;
#pragma unroll
                    for (int i = 0; i < D; ++i) acc = fmaf(gM[l][i], u[i], acc);
                    ge[l] = beta * acc;
                    gb = fmaf(e[l], acc, gb);  // u^T gM' e
                }
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    float pq = 0.f, ph = 0.f, pk = 0.f;
#pragma unroll
                    for (int l = 0; l < CPL; ++l) {
                        pq = fmaf(Mn[l][i], gyv[l], pq);
                        ph = fmaf(gM[l][i], e[l], ph);
                        pk = fmaf(Mp[l][i], ge[l], pk);
                    }
                    part[0][i] = pq;
                    part[1][i] = ph;
                    part[2][i] = pk;
                    part[3][i] = 0.f;
                }
#pragma unroll
                for (int l = 0; l < CPL; ++l)
#pragma unroll
                    for (int i = 0; i < D; ++i) {
                        const float gmb = fmaf(-k[i], ge[l], gM[l][i]);
                        if constexpr (NEED_DYN) part[3][i] = fmaf(gmb, Mp[l][i], part[3][i]);
                        gM[l][i] = a[i] * gmb;
                    }
                float tot[4];
                if constexpr (NEED_DYN) {
                    g.template reduce_scatter<4>(part, tot);
                } else {
                    float part3[3][D];
#pragma unroll
                    for (int v = 0; v < 3; ++v)
#pragma unroll
                        for (int i = 0; i < D; ++i) part3[v][i] = part[v][i];
                    float tot3[3];
                    g.template reduce_scatter<3>(part3, tot3);
                    tot[0] = tot3[0]; tot[1] = tot3[1]; tot[2] = tot3[2]; tot[3] = 0.f;
                }
                const float gq_own = tot[0], h_own = tot[1], mk_own = tot[2], gam_own = tot[3];

                float Ru = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) Ru = fmaf(R[j], u[j], Ru);
                gb = fmaf(-u_own, Ru, gb);
                float trR = 0.f;
                if constexpr (NEED_DYN) {
                    trR = pick(R, own);
                    float two[2] = {gb, trR};
#pragma unroll
                    for (int h = 1; h < D; h <<= 1) {
                        two[0] += g.xor_(two[0], h);
                        two[1] += g.xor_(two[1], h);
                    }
                    gb = two[0];
                    trR = two[1];
                } else {
                    gb = g.allsum(gb);
                }
                const float gs = (s >= floor_) ? -beta * beta * gb : 0.f;
                const float gu_own = beta * h_own - 2.f * beta * Ru + gs * k_own;
                float gu[D];
                g.gather(gu_own, gu);

                // gk = -A Mp ge + gs u + Pbar gu
                float z = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) z = fmaf(Pp[j], a[j] * gu[j], z);
                const float gk3 = fmaf(a_own, z, p * gu_own);
                const float gk_own = fmaf(-a_own, mk_own, fmaf(gs, u_own, gk3));

                // S = R + sym(gu k^T); decay gradient; carry R <- A S A
                float gaP = 0.f, gpk = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) {
                    // rounded products and sum, never contracted to an FMA:
                    // lane i and lane j then form bit-identical S_ij, S_ji
                    const float x = __fadd_rn(__fmul_rn(gu_own, k[j]), __fmul_rn(gu[j], k_own));
                    const float Sj = fmaf(0.5f, x, R[j]);
                    if constexpr (NEED_DYN) {
                        gaP = fmaf(Sj, a[j] * Pp[j], gaP);
                        gpk = fmaf(gu[j], k[j], gpk);
                    }
                    R[j] = (a_own * a[j]) * Sj;
                }

                // outputs
                store_one(A.gk + row * D + own, gk_own);
                store_one(A.gq + row * D + own, gq_own);
                store_vec<CPL>(A.gv + row * M + col0, ge);
                if constexpr (NEED_DYN) {
                    if constexpr (FIXED) {
                        A.ga[row * D + own] = 0.f;
                        if (own == 0) {
                            A.gp[row] = 0.f;
                            A.gr[row] = 0.f;
                        }
                    } else {
                        A.ga[row * D + own] = fmaf(2.f, gaP, gam_own);
                        if (own == 0) {
                            A.gp[row] = trR + gpk;
                            A.gr[row] = gs;
                        }
                    }
                }
            }
#pragma unroll
            for (int l = 0; l < CPL; ++l)
#pragma unroll
                for (int i = 0; i < D; ++i) Mnext[l][i] = Mstart[l][i];
        }
    }
    if constexpr (NEED_INIT) {
        store_mean_cols<D, M>(A.gm0 + chain * D * M, col0, gM);
        store_vec<D>(A.gc0 + chain * D * D + own * D, R);
    }
}

// ===========================================================================
// Host side
// ===========================================================================
thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

inline bool aligned(const void *p, size_t bytes) {
    return p == nullptr || (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

template <int D, int M, int S>
constexpr size_t backward_smem_bytes() {
    return static_cast<size_t>(Launch<D>::kChains) * History<D, M, S>::kFloats * sizeof(float);
}

template <int D, int M, bool FIXED, typename TIn>
int launch_forward(const FwdArgs<TIn> &a, cudaStream_t st) {
    if (a.n == 0) return BSSM_OK;
    const long blocks = (a.n + Launch<D>::kChains - 1) / Launch<D>::kChains;
    if (blocks > 0x7fffffffL) return fail(BSSM_ERR_INVALID, "too many chains");
    forward_kernel<D, M, FIXED, TIn><<<static_cast<unsigned>(blocks), Launch<D>::kThreads, 0, st>>>(a);
    return check_launch("forward_kernel");
}

template <int D, int M, bool FIXED, bool NEED_DYN, bool NEED_INIT, typename TIn>
int launch_backward_impl(const BwdArgs<TIn> &a, cudaStream_t st) {
    constexpr int S = SubChunk<D>::S;
    const long blocks = (a.n + Launch<D>::kChains - 1) / Launch<D>::kChains;
    if (blocks > 0x7fffffffL) return fail(BSSM_ERR_INVALID, "too many chains");
    constexpr size_t smem = backward_smem_bytes<D, M, S>();
    auto kern = backward_kernel<D, M, S, FIXED, NEED_DYN, NEED_INIT, TIn>;
    if (smem > 48 * 1024) {
        cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
        if (err != cudaSuccess)
            return fail(BSSM_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
    }
    kern<<<static_cast<unsigned>(blocks), Launch<D>::kThreads, smem, st>>>(a);
    return check_launch("backward_kernel");
}

template <int D, int M, bool FIXED, typename TIn>
int launch_backward(const BwdArgs<TIn> &a, bool need_dyn, bool need_init, cudaStream_t st) {
    // T = 0 still launches when the initial-state gradients are wanted: the
    // kernel then only maps the final-state gradients onto them.
    if (a.n == 0 || (a.t == 0 && !need_init)) return BSSM_OK;
    if (need_dyn && need_init) return launch_backward_impl<D, M, FIXED, true, true, TIn>(a, st);
    if (need_dyn) return launch_backward_impl<D, M, FIXED, true, false, TIn>(a, st);
    if (need_init) return launch_backward_impl<D, M, FIXED, false, true, TIn>(a, st);
    return launch_backward_impl<D, M, FIXED, false, false, TIn>(a, st);
}

template <int D, int M>
size_t workspace_bytes_t(long n, long t, int chunks) {
    if (n <= 0 || t <= 0 || chunks <= 0) return 0;
    constexpr int S = SubChunk<D>::S;
    const long span = chunks < t ? chunks : t;
    const long nsub_max = (span + S - 1) / S;
    if (nsub_max <= 1) return 0;
    return static_cast<size_t>(n) * static_cast<size_t>(nsub_max - 1) *
           static_cast<size_t>(Slot<D, M>::kChain) * sizeof(float);
}

inline size_t workspace_bytes(int d, int m, long n, long t, int chunks) {
    if (d == 64 && m == 64) return d64_workspace_bytes(n, t, chunks);
    if (m != 8) return 0;
    switch (d) {
        case 1: return workspace_bytes_t<1, 8>(n, t, chunks);
        case 2: return workspace_bytes_t<2, 8>(n, t, chunks);
        case 4: return workspace_bytes_t<4, 8>(n, t, chunks);
        case 8: return workspace_bytes_t<8, 8>(n, t, chunks);
    }
    return 0;
}

inline bool supported(int d, int m) {
    return (m == 8 && (d == 1 || d == 2 || d == 4 || d == 8)) || (d == 64 && m == 64);
}

inline size_t replay_bytes(int d, int m, long n, long t, int chunks) {
    if (n <= 0 || t <= 0 || chunks <= 0) return 0;
    if (d == 64) return 0;  // the D64 backward recomputes each chunk into the workspace
    return static_cast<size_t>(replay_floats(n, t, chunks, d, m)) * sizeof(float);
}

// Kernel families.  Three independently written implementations of the same
// recurrence:
//   chain  -- one thread per chain, history in tensor memory (bssm_chain.cu);
//             needs many chains to fill the GPU (a CTA is 128 chains);
//   staged -- a few lanes per chain, cp.async-staged tiles (bssm_staged.cu);
//   v1     -- D lanes per chain, direct loads (this file).
// Default: chain for large batches, staged below that, v1 where neither
// supports the shape.  BSSM_KERNELS=chain|staged|v1 forces a family (the
// tests run every family against the oracle).
enum Family { kAuto = 0, kChain = 1, kStaged = 2, kV1 = 3, kTile64 = 4 };
constexpr long kChainMinChains = 4096;

// Read at every call (a getenv per launch), so one process can switch.
inline Family forced_family() {
    const char *e = std::getenv("BSSM_KERNELS");
    if (e == nullptr) return kAuto;
    if (std::strcmp(e, "chain") == 0 || std::strcmp(e, "chain1") == 0) return kChain;
    if (std::strcmp(e, "staged") == 0) return kStaged;
    if (std::strcmp(e, "v1") == 0) return kV1;
    return kAuto;
}

template <typename TIn>
Family pick_family(int d, long n, long t, int chunks, bool chain_ok, bool forward) {
    const Family f = forced_family();
    chain_ok = chain_ok && chain_eligible<TIn>(d, n, t, chunks, forward);
    if (f == kV1) return kV1;
    if (f == kChain && chain_ok) return kChain;
    if (f == kAuto && chain_ok && n >= kChainMinChains) return kChain;
    if (staged_supported<TIn>(d)) return kStaged;
    return kV1;
}

// The family the calling thread's last forward / backward launch used.
thread_local int g_last_family = 0;

template <typename TIn>
int forward_dispatch(int d, int fixed, const FwdArgs<TIn> &a, cudaStream_t st) {
    if constexpr (std::is_same_v<TIn, float>) {
        if (d == 64) {
            g_last_family = kTile64;
            return d64_forward(fixed, a, st);
        }
    }
    const Family f = pick_family<TIn>(d, a.n, a.t, a.chunks, true, true);
    g_last_family = f;
    if (f == kChain) return chain_forward<TIn>(d, fixed, a, st);
    if (f == kStaged) return staged_forward<TIn>(d, fixed, a, st);
    switch (d) {
        case 1: return fixed ? launch_forward<1, 8, true>(a, st) : launch_forward<1, 8, false>(a, st);
        case 2: return fixed ? launch_forward<2, 8, true>(a, st) : launch_forward<2, 8, false>(a, st);
        case 4: return fixed ? launch_forward<4, 8, true>(a, st) : launch_forward<4, 8, false>(a, st);
        case 8: return fixed ? launch_forward<8, 8, true>(a, st) : launch_forward<8, 8, false>(a, st);
    }
    return fail(BSSM_ERR_UNSUPPORTED, "key_dim %d", d);
}

template <typename TIn>
int backward_dispatch(int d, int fixed, bool dyn, bool init, const BwdArgs<TIn> &a, cudaStream_t st) {
    if constexpr (std::is_same_v<TIn, float>) {
        if (d == 64) {
            g_last_family = kTile64;
            return d64_backward(fixed, dyn, init, a, st);
        }
    }
    const bool chain_ok = a.rs != nullptr || replay_slots_per_chunk(a.t, a.chunks) == 0;
    const Family f = pick_family<TIn>(d, a.n, a.t, a.chunks, chain_ok, false);
    g_last_family = (f == kStaged && a.t == 0) ? kV1 : f;
    if (f == kChain) return chain_backward<TIn>(d, fixed, dyn, init, a, st);
    if (f == kStaged && a.t > 0) return staged_backward<TIn>(d, fixed, dyn, init, a, st);
    switch (d) {
        case 1: return fixed ? launch_backward<1, 8, true>(a, dyn, init, st)
                             : launch_backward<1, 8, false>(a, dyn, init, st);
        case 2: return fixed ? launch_backward<2, 8, true>(a, dyn, init, st)
                             : launch_backward<2, 8, false>(a, dyn, init, st);
        case 4: return fixed ? launch_backward<4, 8, true>(a, dyn, init, st)
                             : launch_backward<4, 8, false>(a, dyn, init, st);
        case 8: return fixed ? launch_backward<8, 8, true>(a, dyn, init, st)
                             : launch_backward<8, 8, false>(a, dyn, init, st);
    }
    return fail(BSSM_ERR_UNSUPPORTED, "key_dim %d", d);
}

int validate_common(int d, int m, int io_dtype, long n, long t, int chunks, double floor_) {
    if (!supported(d, m))
        return fail(BSSM_ERR_UNSUPPORTED, "(key_dim, value_dim) = (%d, %d) has no kernel; supported: "
                    "(1,8), (2,8), (4,8), (8,8), (64,64)", d, m);
    if (io_dtype != BSSM_F32 && io_dtype != BSSM_BF16)
        return fail(BSSM_ERR_UNSUPPORTED, "io_dtype %d", io_dtype);
    if (d == 64 && io_dtype != BSSM_F32)
        return fail(BSSM_ERR_UNSUPPORTED, "(64, 64) takes float32 keys/values/queries only");
    if (n < 0 || t < 0) return fail(BSSM_ERR_INVALID, "negative size n=%ld t=%ld", n, t);
    if (chunks <= 0) return fail(BSSM_ERR_INVALID, "chunks must be positive (got %d)", chunks);
    if (!(floor_ > 0.0) || floor_ != floor_ || floor_ > 3.0e38)
        return fail(BSSM_ERR_INVALID, "denominator_floor must be finite and positive");
    return BSSM_OK;
}

}  // namespace bssm

// ---------------------------------------------------------------------------
// Allocation-free backward: phase-A scratch in a static device array.
//
// Some callers cannot allocate device memory when they call the backward: a
// host whose allocator owns the whole device budget (a raw allocation would
// bypass it and can fail), a serving loop that cannot take the device-wide
// synchronisation an allocation implies, or a C/FFI host (cgo, JNI, ctypes)
// with no device allocator of its own.  bssm_backward_chunked_noalloc() lets
// them run the recompute-mode backward without passing a workspace: the
// phase-A scratch lives in g_noalloc_scratch, a file-scope array of
// kNoAllocScratchBytes that every GPU loading this library holds until exit.
// ---------------------------------------------------------------------------
namespace bssm {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB per device
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// Device address of g_noalloc_scratch in the current context.  The symbol's
// name in host code is only a host-side stand-in, so the address is looked up
// with cudaGetSymbolAddress (with the device current) once per CUDA context
// and cached under that context: a context created after a device reset gets
// its own lookup instead of a stale address.  Returns nullptr after recording
// an error.
using CtxGetCurrentFn = CUresult (*)(CUcontext *);

static CUcontext current_context() {
    static CtxGetCurrentFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<CtxGetCurrentFn>(nullptr);
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    CUcontext ctx = nullptr;
    if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
    return ctx;
}

static void *noalloc_scratch_current_device() {
    static std::mutex mu;
    static std::unordered_map<CUcontext, void *> cache;
    int dev = -1;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) {
        fail(BSSM_ERR_CUDA, "noalloc backward: cudaGetDevice: %s", cudaGetErrorString(err));
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    CUcontext ctx = current_context();
    if (ctx != nullptr) {
        auto it = cache.find(ctx);
        if (it != cache.end()) return it->second;
    }
    void *ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);  // also makes the device's context current
    if (err != cudaSuccess || ptr == nullptr) {
        fail(BSSM_ERR_CUDA, "noalloc backward: cudaGetSymbolAddress on device %d: %s", dev,
             cudaGetErrorString(err));
        return nullptr;
    }
    ctx = current_context();
    if (ctx == nullptr) {
        fail(BSSM_ERR_CUDA, "noalloc backward: no current context on device %d", dev);
        return nullptr;
    }
    cache[ctx] = ptr;
    return ptr;
}

}  // namespace bssm

using namespace bssm;

extern "C" {

const char *bssm_last_error(void) { return g_last_error.c_str(); }

int bssm_debug_last_family(void) { return bssm::g_last_family; }

int bssm_version(void) { return 10000; }

int bssm_forward_chunked_ex(int key_dim, int value_dim, int io_dtype, int fixed, const void *keys,
                            const void *values, const void *queries, const float *decay,
                            const float *process, const float *observation, const float *mean0,
                            const float *cov0, float *out, float *mean_final, float *cov_final,
                            float *boundary_mean, float *boundary_cov, float *replay_states,
                            size_t replay_states_bytes, long n, long t, int chunks,
                            double denominator_floor, void *stream) {
    int rc = validate_common(key_dim, value_dim, io_dtype, n, t, chunks, denominator_floor);
    if (rc) return rc;
    if (n == 0) {
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!mean_final || !cov_final || !boundary_mean || !boundary_cov)
        return fail(BSSM_ERR_INVALID, "forward: null output pointer");
    const size_t rs_need = replay_bytes(key_dim, value_dim, n, t, chunks);
    if (rs_need == 0) replay_states = nullptr;  // nothing to save (chunks <= the replay span)
    if (replay_states != nullptr && replay_states_bytes < rs_need)
        return fail(BSSM_ERR_WORKSPACE, "forward: replay_states of %zu bytes required (got %zu)", rs_need,
                    replay_states_bytes);
    if (t > 0 && (!keys || !values || !queries || !out))
        return fail(BSSM_ERR_INVALID, "forward: null keys/values/queries/out");
    if (!fixed && t > 0 && (!decay || !process || !observation))
        return fail(BSSM_ERR_INVALID, "forward: decay/process/observation required unless fixed");
    // every tensor is moved with up-to-16-byte vector accesses and cp.async:
    // require 16-byte aligned base pointers (any fresh CUDA allocation is)
    const void *ptrs[] = {keys, values, queries, decay, process, observation, mean0, cov0, out,
                          mean_final, cov_final, boundary_mean, boundary_cov, replay_states};
    for (const void *p : ptrs)
        if (!aligned(p, 16)) return fail(BSSM_ERR_ALIGNMENT, "forward: pointer %p is not 16-byte aligned", p);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const float fl = static_cast<float>(denominator_floor);
    if (io_dtype == BSSM_F32) {
        FwdArgs<float> a{static_cast<const float *>(keys), static_cast<const float *>(values),
                         static_cast<const float *>(queries), decay, process, observation, mean0, cov0,
                         out, mean_final, cov_final, boundary_mean, boundary_cov, replay_states, n, t,
                         chunks, fl};
        return forward_dispatch(key_dim, fixed, a, st);
    }
    FwdArgs<__nv_bfloat16> a{static_cast<const __nv_bfloat16 *>(keys),
                             static_cast<const __nv_bfloat16 *>(values),
                             static_cast<const __nv_bfloat16 *>(queries), decay, process, observation,
                             mean0, cov0, out, mean_final, cov_final, boundary_mean, boundary_cov,
                             replay_states, n, t, chunks, fl};
    return forward_dispatch(key_dim, fixed, a, st);
}

size_t bssm_replay_states_bytes(int key_dim, int value_dim, long n, long t, int chunks) {
    if (!supported(key_dim, value_dim)) return 0;
    return replay_bytes(key_dim, value_dim, n, t, chunks);
}

size_t bssm_backward_workspace_bytes(int key_dim, int value_dim, long n, long t, int chunks) {
    if (!supported(key_dim, value_dim)) return 0;
    return workspace_bytes(key_dim, value_dim, n, t, chunks);
}

int bssm_backward_chunked_ex(int key_dim, int value_dim, int io_dtype, int fixed, int need_dynamics,
                             int need_initial, const void *keys, const void *values,
                             const void *queries, const float *decay, const float *process,
                             const float *observation, const float *mean0, const float *cov0,
                             const float *boundary_mean, const float *boundary_cov,
                             const float *replay_states, size_t replay_states_bytes,
                             const float *grad_out, const float *grad_mean_final,
                             const float *grad_cov_final, void *grad_keys, void *grad_values,
                             void *grad_queries, float *grad_decay, float *grad_process,
                             float *grad_observation, float *grad_mean0, float *grad_cov0,
                             void *workspace, size_t workspace_bytes_, long n, long t, int chunks,
                             double denominator_floor, void *stream) {
    (void)mean0;
    (void)cov0;
    int rc = validate_common(key_dim, value_dim, io_dtype, n, t, chunks, denominator_floor);
    if (rc) return rc;
    const bool dyn = need_dynamics != 0, init = need_initial != 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (n == 0) {
        g_last_error.clear();
        return BSSM_OK;
    }
    if (init && (!grad_mean0 || !grad_cov0))
        return fail(BSSM_ERR_INVALID, "backward: need_initial requires grad_mean0/grad_cov0");
    if (t == 0 && !init) {
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!boundary_mean || !boundary_cov)
        return fail(BSSM_ERR_INVALID, "backward: null boundary state pointer");
    if (t > 0 && (!keys || !values || !queries || !grad_keys || !grad_values || !grad_queries))
        return fail(BSSM_ERR_INVALID, "backward: null input or gradient pointer");
    if (!fixed && t > 0 && (!decay || !process || !observation))
        return fail(BSSM_ERR_INVALID, "backward: decay/process/observation required unless fixed");
    if (dyn && t > 0 && (!grad_decay || !grad_process || !grad_observation))
        return fail(BSSM_ERR_INVALID, "backward: need_dynamics requires grad_decay/process/observation");
    const size_t rs_need = replay_bytes(key_dim, value_dim, n, t, chunks);
    if (rs_need == 0) replay_states = nullptr;
    if (replay_states != nullptr && replay_states_bytes < rs_need)
        return fail(BSSM_ERR_WORKSPACE, "backward: replay_states of %zu bytes required (got %zu)", rs_need,
                    replay_states_bytes);
    // the phase-A workspace is needed only when the replay states were not saved
    const size_t need = replay_states ? 0 : workspace_bytes(key_dim, value_dim, n, t, chunks);
    if (need > 0 && (workspace == nullptr || workspace_bytes_ < need))
        return fail(BSSM_ERR_WORKSPACE, "backward: workspace of %zu bytes required (got %zu)", need,
                    workspace_bytes_);
    const void *ptrs[] = {keys, values, queries, decay, process, observation, boundary_mean,
                          boundary_cov, replay_states, grad_out, grad_mean_final, grad_cov_final,
                          grad_keys, grad_values, grad_queries, grad_decay, grad_process,
                          grad_observation, grad_mean0, grad_cov0, workspace};
    for (const void *p : ptrs)
        if (!aligned(p, 16)) return fail(BSSM_ERR_ALIGNMENT, "backward: pointer %p is not 16-byte aligned", p);
    const float fl = static_cast<float>(denominator_floor);
    float *ws = static_cast<float *>(workspace);
    if (io_dtype == BSSM_F32) {
        BwdArgs<float> a{static_cast<const float *>(keys), static_cast<const float *>(values),
                         static_cast<const float *>(queries), decay, process, observation, mean0, cov0,
                         boundary_mean, boundary_cov, grad_out, grad_mean_final, grad_cov_final,
                         static_cast<float *>(grad_keys), static_cast<float *>(grad_values),
                         static_cast<float *>(grad_queries), grad_decay, grad_process, grad_observation,
                         grad_mean0, grad_cov0, ws, replay_states, n, t, chunks, fl};
        return backward_dispatch(key_dim, fixed, dyn, init, a, st);
    }
    BwdArgs<__nv_bfloat16> a{static_cast<const __nv_bfloat16 *>(keys),
                             static_cast<const __nv_bfloat16 *>(values),
                             static_cast<const __nv_bfloat16 *>(queries), decay, process, observation,
                             mean0, cov0, boundary_mean, boundary_cov, grad_out, grad_mean_final,
                             grad_cov_final, static_cast<__nv_bfloat16 *>(grad_keys),
                             static_cast<__nv_bfloat16 *>(grad_values),
                             static_cast<__nv_bfloat16 *>(grad_queries), grad_decay, grad_process,
                             grad_observation, grad_mean0, grad_cov0, ws, replay_states, n, t, chunks, fl};
    return backward_dispatch(key_dim, fixed, dyn, init, a, st);
}

// ---- reference-named float32 wrappers ---------------------------------------
#define BSSM_DEFINE_DIM(DN, MN)                                                                        \
    int bssm_d##DN##_forward_chunked(const float *keys, const float *values, const float *queries,   \
                                     const float *decay, const float *process,                     \
                                     const float *observation, const float *mean0,                 \
                                     const float *cov0, float *out, float *mean_final,             \
                                     float *cov_final, float *boundary_mean, float *boundary_cov,  \
                                     long n, long t, int chunks, double denominator_floor,         \
                                     void *stream) {                                               \
        return bssm_forward_chunked_ex(DN, MN, BSSM_F32, 0, keys, values, queries, decay, process,  \
                                       observation, mean0, cov0, out, mean_final, cov_final,       \
                                       boundary_mean, boundary_cov, nullptr, 0, n, t, chunks,      \
                                       denominator_floor, stream);                                 \
    }                                                                                              \
    int bssm_d##DN##_forward_chunked_fixed(const float *keys, const float *values,                 \
                                           const float *queries, const float *decay,               \
                                           const float *process, const float *observation,         \
                                           const float *mean0, const float *cov0, float *out,      \
                                           float *mean_final, float *cov_final,                    \
                                           float *boundary_mean, float *boundary_cov, long n,      \
                                           long t, int chunks, double denominator_floor,           \
                                           void *stream) {                                         \
        return bssm_forward_chunked_ex(DN, MN, BSSM_F32, 1, keys, values, queries, decay, process,  \
                                       observation, mean0, cov0, out, mean_final, cov_final,       \
                                       boundary_mean, boundary_cov, nullptr, 0, n, t, chunks,      \
                                       denominator_floor, stream);                                 \
    }                                                                                              \
    int bssm_d##DN##_backward_chunked(                                                             \
        const float *keys, const float *values, const float *queries, const float *decay,          \
        const float *process, const float *observation, const float *mean0, const float *cov0,     \
        const float *boundary_mean, const float *boundary_cov, const float *grad_out,              \
        const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,               \
        float *grad_values, float *grad_queries, float *grad_decay, float *grad_process,           \
        float *grad_observation, float *grad_mean0, float *grad_cov0, void *workspace,             \
        size_t workspace_bytes, long n, long t, int chunks, double denominator_floor,              \
        void *stream) {                                                                            \
        return bssm_backward_chunked_ex(DN, MN, BSSM_F32, 0, 1, 1, keys, values, queries, decay,    \
                                        process, observation, mean0, cov0, boundary_mean,          \
                                        boundary_cov, nullptr, 0, grad_out, grad_mean_final,       \
                                        grad_cov_final,                                            \
                                        grad_keys, grad_values, grad_queries, grad_decay,          \
                                        grad_process, grad_observation, grad_mean0, grad_cov0,     \
                                        workspace, workspace_bytes, n, t, chunks,                  \
                                        denominator_floor, stream);                                \
    }                                                                                              \
    int bssm_d##DN##_backward_chunked_lean(                                                        \
        const float *keys, const float *values, const float *queries, const float *decay,          \
        const float *process, const float *observation, const float *mean0, const float *cov0,     \
        const float *boundary_mean, const float *boundary_cov, const float *grad_out,              \
        const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,               \
        float *grad_values, float *grad_queries, void *workspace, size_t workspace_bytes, long n,  \
        long t, int chunks, double denominator_floor, void *stream) {                              \
        return bssm_backward_chunked_ex(DN, MN, BSSM_F32, 0, 0, 0, keys, values, queries, decay,    \
                                        process, observation, mean0, cov0, boundary_mean,          \
                                        boundary_cov, nullptr, 0, grad_out, grad_mean_final,       \
                                        grad_cov_final,                                            \
                                        grad_keys, grad_values, grad_queries, nullptr, nullptr,    \
                                        nullptr, nullptr, nullptr, workspace, workspace_bytes, n,  \
                                        t, chunks, denominator_floor, stream);                     \
    }                                                                                              \
    int bssm_d##DN##_backward_chunked_fixed(                                                       \
        const float *keys, const float *values, const float *queries, const float *decay,          \
        const float *process, const float *observation, const float *mean0, const float *cov0,     \
        const float *boundary_mean, const float *boundary_cov, const float *grad_out,              \
        const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,               \
        float *grad_values, float *grad_queries, float *grad_decay, float *grad_process,           \
        float *grad_observation, float *grad_mean0, float *grad_cov0, void *workspace,             \
        size_t workspace_bytes, long n, long t, int chunks, double denominator_floor,              \
        void *stream) {                                                                            \
        return bssm_backward_chunked_ex(DN, MN, BSSM_F32, 1, 1, 1, keys, values, queries, decay,    \
                                        process, observation, mean0, cov0, boundary_mean,          \
                                        boundary_cov, nullptr, 0, grad_out, grad_mean_final,       \
                                        grad_cov_final,                                            \
                                        grad_keys, grad_values, grad_queries, grad_decay,          \
                                        grad_process, grad_observation, grad_mean0, grad_cov0,     \
                                        workspace, workspace_bytes, n, t, chunks,                  \
                                        denominator_floor, stream);                                \
    }                                                                                              \
    int bssm_d##DN##_backward_chunked_lean_fixed(                                                  \
        const float *keys, const float *values, const float *queries, const float *decay,          \
        const float *process, const float *observation, const float *mean0, const float *cov0,     \
        const float *boundary_mean, const float *boundary_cov, const float *grad_out,              \
        const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,               \
        float *grad_values, float *grad_queries, void *workspace, size_t workspace_bytes, long n,  \
        long t, int chunks, double denominator_floor, void *stream) {                              \
        return bssm_backward_chunked_ex(DN, MN, BSSM_F32, 1, 0, 0, keys, values, queries, decay,    \
                                        process, observation, mean0, cov0, boundary_mean,          \
                                        boundary_cov, nullptr, 0, grad_out, grad_mean_final,       \
                                        grad_cov_final,                                            \
                                        grad_keys, grad_values, grad_queries, nullptr, nullptr,    \
                                        nullptr, nullptr, nullptr, workspace, workspace_bytes, n,  \
                                        t, chunks, denominator_floor, stream);                     \
    }

BSSM_DEFINE_DIM(1, 8)
BSSM_DEFINE_DIM(2, 8)
BSSM_DEFINE_DIM(4, 8)
BSSM_DEFINE_DIM(8, 8)
BSSM_DEFINE_DIM(64, 64)

int bssm_d2_backward_chunked_noinitial(
    const float *keys, const float *values, const float *queries, const float *decay,
    const float *process, const float *observation, const float *mean0, const float *cov0,
    const float *boundary_mean, const float *boundary_cov, const float *grad_out,
    const float *grad_mean_final, const float *grad_cov_final, float *grad_keys, float *grad_values,
    float *grad_queries, float *grad_decay, float *grad_process, float *grad_observation,
    void *workspace, size_t workspace_bytes, long n, long t, int chunks, double denominator_floor,
    void *stream) {
    return bssm_backward_chunked_ex(2, 8, BSSM_F32, 0, 1, 0, keys, values, queries, decay, process,
                                    observation, mean0, cov0, boundary_mean, boundary_cov, nullptr, 0,
                                    grad_out, grad_mean_final, grad_cov_final, grad_keys, grad_values,
                                    grad_queries, grad_decay, grad_process, grad_observation,
                                    nullptr, nullptr, workspace, workspace_bytes, n, t, chunks,
                                    denominator_floor, stream);
}

int bssm_d2_backward_chunked_noinitial_fixed(
    const float *keys, const float *values, const float *queries, const float *decay,
    const float *process, const float *observation, const float *mean0, const float *cov0,
    const float *boundary_mean, const float *boundary_cov, const float *grad_out,
    const float *grad_mean_final, const float *grad_cov_final, float *grad_keys, float *grad_values,
    float *grad_queries, float *grad_decay, float *grad_process, float *grad_observation,
    void *workspace, size_t workspace_bytes, long n, long t, int chunks, double denominator_floor,
    void *stream) {
    return bssm_backward_chunked_ex(2, 8, BSSM_F32, 1, 1, 0, keys, values, queries, decay, process,
                                    observation, mean0, cov0, boundary_mean, boundary_cov, nullptr, 0,
                                    grad_out, grad_mean_final, grad_cov_final, grad_keys, grad_values,
                                    grad_queries, grad_decay, grad_process, grad_observation,
                                    nullptr, nullptr, workspace, workspace_bytes, n, t, chunks,
                                    denominator_floor, stream);
}

size_t bssm_backward_noalloc_max_scratch_bytes(void) { return kNoAllocScratchBytes; }

int bssm_backward_chunked_noalloc(int key_dim, int value_dim, int io_dtype, int fixed,
                                  int need_dynamics, int need_initial, const void *keys,
                                  const void *values, const void *queries, const float *decay,
                                  const float *process, const float *observation,
                                  const float *mean0, const float *cov0,
                                  const float *boundary_mean, const float *boundary_cov,
                                  const float *grad_out, const float *grad_mean_final,
                                  const float *grad_cov_final, void *grad_keys, void *grad_values,
                                  void *grad_queries, float *grad_decay, float *grad_process,
                                  float *grad_observation, float *grad_mean0, float *grad_cov0,
                                  long n, long t, int chunks, double denominator_floor, void *stream) {
    int rc = validate_common(key_dim, value_dim, io_dtype, n, t, chunks, denominator_floor);
    if (rc) return rc;
    const size_t need = workspace_bytes(key_dim, value_dim, n, t, chunks);
    if (need > kNoAllocScratchBytes)
        return fail(BSSM_ERR_WORKSPACE,
                    "noalloc backward: this problem needs %zu bytes of scratch but the static scratch "
                    "holds %zu (n=%ld, t=%ld, chunks=%d); use bssm_backward_chunked_ex with a "
                    "caller-provided workspace or the forward's replay states",
                    need, kNoAllocScratchBytes, n, t, chunks);
    void *scratch = nullptr;
    if (need > 0) {
        scratch = noalloc_scratch_current_device();
        if (scratch == nullptr) return BSSM_ERR_CUDA;
    }
    // the scratch is written before it is read inside one launch: no clearing
    return bssm_backward_chunked_ex(key_dim, value_dim, io_dtype, fixed, need_dynamics, need_initial, keys,
                                    values, queries, decay, process, observation, mean0, cov0,
                                    boundary_mean, boundary_cov, nullptr, 0, grad_out, grad_mean_final,
                                    grad_cov_final, grad_keys, grad_values, grad_queries, grad_decay,
                                    grad_process, grad_observation, grad_mean0, grad_cov0, scratch,
                                    need > 0 ? kNoAllocScratchBytes : 0, n, t, chunks, denominator_floor,
                                    stream);
}

}  // extern "C"
