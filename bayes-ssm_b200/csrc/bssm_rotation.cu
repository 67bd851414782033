// bssm_rotation.cu -- the chunked recurrence with rotation dynamics.
//
// The reference has no kernel for this path: bayes_ssm/bayesian_layer.py
// (:254-340 and the make_rotation_dynamics / make_rotation_process_covariances
// helpers) builds dense block-diagonal transitions and per-pair process
// covariances and runs its dense recurrence.  Here the same model runs on
// the GPU with the 2 x 2 block structure used directly:
//
//   A = blockdiag(A_m),  A_m = [[c_m, -s_m], [s_m, c_m]]  (c = rho cos theta,
//       s = rho sin theta, the caller's damped rotation),
//   Q = blockdiag(diag(q_m, 0)),
//   P' = A P A^T + Q, M' = A M, then the same gain / update / readout as the
//   diagonal kernels (bayesian_layer.py:153-181).
//
// D lanes serve one chain (D = 2, 4, 8; M = 8): lane i owns covariance row i
// and M / D mean columns.  Row i of A P A^T needs only rows i and i ^ 1 of P
// (one butterfly with the partner lane), and is summed in a fixed grouping
// that makes entries (i, j) and (j, i) bit-identical, so the covariance stays
// exactly symmetric.  The backward is recompute mode: per chunk, replay it
// saving each 4-token sub-chunk's start state to the caller's workspace, then
// per sub-chunk replay with the history in shared memory (thread-private
// slots) and run the reverse step.  It returns the gradients of c and s per
// pair; the caller's autograd carries them to the radii and angles.
#include <cuda_runtime.h>

#include <cstdint>

#include "bayes_ssm_b200.h"
#include "bssm_common.cuh"
#include "bssm_internal.h"

namespace bssm {
namespace rot {

constexpr int kThreads = 128;
constexpr int kSub = 4;
// CTAs per SM the backward's registers are sized for.  At config 3's shape
// (16,384 chains at D8: 1,024 CTAs) four per SM run the launch in two waves
// where three (166 registers, no spills) took three: 8.00 against 8.36 ms per
// API step, with 52 bytes spilled; three per SM forced: 8.73 ms.  Loading the
// chunk replay's tokens one ahead, as the forward does, was slower here (6.67 ms
// at four CTAs, spilling more; 6.98 at three, against 6.51), and so was an L2
// prefetch of each chain's next 4-token block in both kernels (6.66 against
// 6.52): at four CTAs per SM the loads' latency is not what binds.
#ifndef BSSM_ROT_BWD_MINB
#define BSSM_ROT_BWD_MINB 4
#endif
// The forward's launch bounds (by default the block size alone).  Before its
// one-token prefetch (96 registers, five CTAs per SM), eight or six per SM (64 /
// 80 registers, with spills) did not help: 7.95-8.18 and 8.11 against 7.97 ms
// per API step.  The prefetch (128 registers): 6.66 -> 6.48 ms.
#ifdef BSSM_ROT_FWD_MINB
#define BSSM_ROT_FWD_BOUNDS __launch_bounds__(kThreads, BSSM_ROT_FWD_MINB)
#else
#define BSSM_ROT_FWD_BOUNDS __launch_bounds__(kThreads)
#endif

struct Args {
    const float *keys, *values, *queries;  // [N,T,D], [N,T,M], [N,T,D]
    const float *cosines, *sines;          // [N,T,D/2]: rho cos, rho sin
    const float *process;                  // [N,T,D/2]: per-pair variance on the even coordinate
    const float *observation;              // [N,T]
    const float *mean0, *cov0;             // [N,D,M], [N,D,D] (NULL: zeros, identity)
    float *out, *mean_final, *cov_final;   // forward outputs
    float *bmean, *bcov;                   // [N,NB+1,D,M], [N,NB+1,D,D]
    const float *gy, *gmf, *gcf;           // backward inputs (NULL = zeros)
    float *gk, *gv, *gq, *gcos, *gsin, *gproc, *gobs, *gm0, *gc0;
    float *ws;
    long n, t;
    int chunks;
    float floor;
};

template <int D, int M>
struct Tok {
    static constexpr int J = D / 2, CPL = M / D;
    float k[D], q[D], c[J], s[J], qp[J], v[CPL], gy[CPL];
    float r;
};

template <int D, int M, bool WANT_GY>
__device__ __forceinline__ void load_tok(Tok<D, M> &tk, const Args &A, long row, int col0) {
    constexpr int J = D / 2, CPL = M / D;
    load_vec<D>(A.keys + row * D, tk.k);
    load_vec<D>(A.queries + row * D, tk.q);
    load_vec<J>(A.cosines + row * J, tk.c);
    load_vec<J>(A.sines + row * J, tk.s);
    load_vec<J>(A.process + row * J, tk.qp);
    load_vec<CPL>(A.values + row * M + col0, tk.v);
    tk.r = __ldg(A.observation + row);
    if constexpr (WANT_GY) {
        if (A.gy != nullptr) {
            load_vec<CPL>(A.gy + row * M + col0, tk.gy);
        } else {
#pragma unroll
            for (int l = 0; l < CPL; ++l) tk.gy[l] = 0.f;
        }
    }
}

// Entries of row i of A (i ^ 1 is the partner): diag A_ii = c, off A_i,i^1 =
// -s for even i, +s for odd i.
template <int D, int M>
__device__ __forceinline__ float a_diag(const Tok<D, M> &tk, int i) { return tk.c[i >> 1]; }
template <int D, int M>
__device__ __forceinline__ float a_off(const Tok<D, M> &tk, int i) {
    return (i & 1) ? tk.s[i >> 1] : -tk.s[i >> 1];
}

// Row `own` of B X B^T (X symmetric, B block-diagonal 2 x 2) from rows own
// (x) and own ^ 1 (xp) of X, with bi = (B_own,own, B_own,own^1) and the
// per-row entries of B given by (bd[j], bo[j]) = (B_jj, B_j,j^1).  The sum is
// grouped as ((T1 + T4) + (T2 + T3)) with non-contracted products, so lane j
// computing entry (j, own) gets the same bits.
template <int D>
__device__ __forceinline__ void congruence_row(const float (&x)[D], const float (&xp)[D], float bii, float bio,
                                               const float (&bd)[D], const float (&bo)[D], float (&o)[D]) {
#pragma unroll
    for (int j = 0; j < D; ++j) {
        const int pj = j ^ 1;
        const float t1 = __fmul_rn(__fmul_rn(bii, bd[j]), x[j]);
        const float t4 = __fmul_rn(__fmul_rn(bio, bo[j]), xp[pj]);
        const float t2 = __fmul_rn(__fmul_rn(bio, bd[j]), xp[j]);
        const float t3 = __fmul_rn(__fmul_rn(bii, bo[j]), x[pj]);
        o[j] = __fadd_rn(__fadd_rn(t1, t4), __fadd_rn(t2, t3));
    }
}

// Rows of A (as bd, bo per row j) and of A^T (B = A^T: B_jj = A_jj,
// B_j,j^1 = A_j^1,j = -A_j,j^1).
template <int D, int M>
__device__ __forceinline__ void a_rows(const Tok<D, M> &tk, float (&bd)[D], float (&bo)[D], bool transpose) {
#pragma unroll
    for (int j = 0; j < D; ++j) {
        bd[j] = a_diag(tk, j);
        bo[j] = transpose ? -a_off(tk, j) : a_off(tk, j);
    }
}

// Q: the pair's variance on the even coordinate of the diagonal.
template <int D>
__device__ __forceinline__ void add_pair_noise(float (&row)[D], const float (&qp)[D / 2], int own) {
#pragma unroll
    for (int j = 0; j < D; j += 2)
        if (j == own) row[j] = __fadd_rn(row[j], qp[j >> 1]);
}

template <int D, int M>
struct Step {
    float pbar[D];   // row own of the predicted covariance
    float u[D];      // gain, all rows
    float e[M / D];  // innovation at the lane's columns
    float u_own, beta, s;
};

// One predict / update step of the lane's slice, in place.
template <int D, int M>
__device__ __forceinline__ void fwd_step(const LaneGroup<D> &g, const Tok<D, M> &tk, float (&Mc)[M / D][D],
                                         float (&P)[D], float floor_, Step<D, M> &o) {
    constexpr int CPL = M / D;
    const int own = g.sub;
    float Pq[D];
#pragma unroll
    for (int j = 0; j < D; ++j) Pq[j] = g.xor_(P[j], 1);
    float bd[D], bo[D];
    a_rows(tk, bd, bo, false);
    congruence_row<D>(P, Pq, pick(bd, own), pick(bo, own), bd, bo, o.pbar);
    add_pair_noise(o.pbar, tk.qp, own);
    float z = 0.f;
#pragma unroll
    for (int j = 0; j < D; ++j) z = fmaf(o.pbar[j], tk.k[j], z);
    const float u_own = z;
    g.gather(u_own, o.u);
    o.u_own = u_own;
    float s = tk.r;
#pragma unroll
    for (int j = 0; j < D; ++j) s = fmaf(tk.k[j], o.u[j], s);
    o.s = s;
    const float beta = 1.0f / (s < floor_ ? floor_ : s);
    o.beta = beta;
    // mean: M_bar = A M (rows i and i ^ 1 of every column are in the lane)
#pragma unroll
    for (int l = 0; l < CPL; ++l) {
        float mb[D];
#pragma unroll
        for (int i = 0; i < D; ++i) mb[i] = fmaf(a_diag(tk, i), Mc[l][i], a_off(tk, i) * Mc[l][i ^ 1]);
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < D; ++i) acc = fmaf(mb[i], tk.k[i], acc);
        o.e[l] = tk.v[l] - acc;
        const float be = beta * o.e[l];
#pragma unroll
        for (int i = 0; i < D; ++i) Mc[l][i] = fmaf(be, o.u[i], mb[i]);
    }
#pragma unroll
    for (int j = 0; j < D; ++j) P[j] = fmaf(-beta, u_own * o.u[j], o.pbar[j]);
}

template <int D, int M>
__device__ __forceinline__ void load_state(const float *mean, const float *cov, int own, int col0,
                                           float (&Mc)[M / D][D], float (&P)[D]) {
    constexpr int CPL = M / D;
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int l = 0; l < CPL; ++l) Mc[l][i] = mean ? mean[i * M + col0 + l] : 0.f;
#pragma unroll
    for (int j = 0; j < D; ++j) P[j] = cov ? 0.5f * (cov[own * D + j] + cov[j * D + own]) : (j == own ? 1.f : 0.f);
}
template <int D, int M>
__device__ __forceinline__ void store_state(float *mean, float *cov, int own, int col0, const float (&Mc)[M / D][D],
                                            const float (&P)[D]) {
    constexpr int CPL = M / D;
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int l = 0; l < CPL; ++l) mean[i * M + col0 + l] = Mc[l][i];
#pragma unroll
    for (int j = 0; j < D; ++j) cov[own * D + j] = P[j];
}

// ---------------------------------------------------------------------------
template <int D, int M>
__global__ void BSSM_ROT_FWD_BOUNDS rot_forward(const Args A) {
    constexpr int CPL = M / D;
    const LaneGroup<D> g;
    const long chain = (static_cast<long>(blockIdx.x) * kThreads + threadIdx.x) / D;
    if (chain >= A.n) return;  // whole lane groups retire together
    const int own = g.sub, col0 = own * CPL;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;
    float Mc[CPL][D], P[D];
    load_state<D, M>(A.mean0 ? A.mean0 + chain * D * M : nullptr, A.cov0 ? A.cov0 + chain * D * D : nullptr, own,
                     col0, Mc, P);
    float *bm = A.bmean + chain * (nb + 1) * D * M;
    float *bc = A.bcov + chain * (nb + 1) * D * D;
    store_state<D, M>(bm, bc, own, col0, Mc, P);
    Tok<D, M> nx;  // the next token's inputs, loaded one token ahead
    if (T > 0) load_tok<D, M, false>(nx, A, chain * T, col0);
    for (long ti = 0; ti < T; ++ti) {
        const long row = chain * T + ti;
        const Tok<D, M> tk = nx;
        if (ti + 1 < T) load_tok<D, M, false>(nx, A, row + 1, col0);
        Step<D, M> o;
        fwd_step<D, M>(g, tk, Mc, P, A.floor, o);
#pragma unroll
        for (int l = 0; l < CPL; ++l) {
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < D; ++i) acc = fmaf(Mc[l][i], tk.q[i], acc);
            A.out[row * M + col0 + l] = acc;
        }
        if ((ti + 1) % L == 0 || ti + 1 == T) {
            const long b = (ti + L) / L;
            store_state<D, M>(bm + b * D * M, bc + b * D * D, own, col0, Mc, P);
        }
    }
    store_state<D, M>(A.mean_final + chain * D * M, A.cov_final + chain * D * D, own, col0, Mc, P);
}

// Per-lane history floats of one token: covariance row, mean columns, the
// lane's innovation entries, its gain entry, beta and s.
template <int D, int M>
struct Hist {
    static constexpr int CPL = M / D;
    static constexpr int kP = 0, kM = D, kE = D + M, kU = kE + CPL, kB = kU + 1, kS = kB + 1;
    static constexpr int kFloats = kS + 1;
};

template <int D, int M, bool NEED_INIT>
__global__ void __launch_bounds__(kThreads, BSSM_ROT_BWD_MINB) rot_backward(const Args A) {
    constexpr int CPL = M / D, J = D / 2;
    using H = Hist<D, M>;
    __shared__ float hist[kSub * H::kFloats * kThreads];
    const LaneGroup<D> g;
    const int tid = threadIdx.x;
    const long chain = (static_cast<long>(blockIdx.x) * kThreads + tid) / D;
    if (chain >= A.n) return;
    const int own = g.sub, col0 = own * CPL, pown = own ^ 1;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;
    const int nsub_max = (static_cast<int>(L < T ? L : T) + kSub - 1) / kSub;
    const int lane_state = D + M;  // floats of a saved state per lane
    float *const ws = A.ws + (chain * static_cast<long>(nsub_max > 1 ? nsub_max - 1 : 0) * D + own) * lane_state;
    const long ws_stride = static_cast<long>(D) * lane_state;  // one saved state of the chain
    auto hx = [&](int x, int f) -> float & { return hist[(x * H::kFloats + f) * kThreads + tid]; };

    float gM[CPL][D], R[D];
#pragma unroll
    for (int i = 0; i < D; ++i)
#pragma unroll
        for (int l = 0; l < CPL; ++l) gM[l][i] = A.gmf ? A.gmf[chain * D * M + i * M + col0 + l] : 0.f;
#pragma unroll
    for (int j = 0; j < D; ++j) {
        const float *gc = A.gcf ? A.gcf + chain * D * D : nullptr;
        R[j] = gc ? 0.5f * (gc[own * D + j] + gc[j * D + own]) : 0.f;
    }

    for (long ci = nb - 1; ci >= 0; --ci) {
        const long t0 = ci * L;
        const int len = static_cast<int>(L < T - t0 ? L : T - t0);
        const int nsub = (len + kSub - 1) / kSub;
        const float *bm = A.bmean + (chain * (nb + 1) + ci) * D * M;
        const float *bc = A.bcov + (chain * (nb + 1) + ci) * D * D;
        float Mc[CPL][D], P[D];
        if (nsub > 1) {  // phase A: sub-chunk start states
            load_state<D, M>(bm, bc, own, col0, Mc, P);
            for (int li = 0; li < (nsub - 1) * kSub; ++li) {
                Tok<D, M> tk;
                load_tok<D, M, false>(tk, A, chain * T + t0 + li, col0);
                Step<D, M> o;
                fwd_step<D, M>(g, tk, Mc, P, A.floor, o);
                if ((li + 1) % kSub == 0) {
                    float *dst = ws + static_cast<long>((li + 1) / kSub - 1) * ws_stride;
#pragma unroll
                    for (int j = 0; j < D; ++j) dst[j] = P[j];
#pragma unroll
                    for (int l = 0; l < CPL; ++l)
#pragma unroll
                        for (int i = 0; i < D; ++i) dst[D + l * D + i] = Mc[l][i];
                }
            }
        }
        for (int sb = nsub - 1; sb >= 0; --sb) {
            const int s0 = sb * kSub;
            const int slen = len - s0 < kSub ? len - s0 : kSub;
            if (sb == 0) {
                load_state<D, M>(bm, bc, own, col0, Mc, P);
            } else {
                const float *src = ws + static_cast<long>(sb - 1) * ws_stride;
#pragma unroll
                for (int j = 0; j < D; ++j) P[j] = src[j];
#pragma unroll
                for (int l = 0; l < CPL; ++l)
#pragma unroll
                    for (int i = 0; i < D; ++i) Mc[l][i] = src[D + l * D + i];
            }
            // replay with history (thread-private shared-memory slots)
            for (int x = 0; x < slen; ++x) {
                Tok<D, M> tk;
                load_tok<D, M, false>(tk, A, chain * T + t0 + s0 + x, col0);
#pragma unroll
                for (int j = 0; j < D; ++j) hx(x, H::kP + j) = P[j];
#pragma unroll
                for (int l = 0; l < CPL; ++l)
#pragma unroll
                    for (int i = 0; i < D; ++i) hx(x, H::kM + l * D + i) = Mc[l][i];
                Step<D, M> o;
                fwd_step<D, M>(g, tk, Mc, P, A.floor, o);
#pragma unroll
                for (int l = 0; l < CPL; ++l) hx(x, H::kE + l) = o.e[l];
                hx(x, H::kU) = o.u_own;
                hx(x, H::kB) = o.beta;
                hx(x, H::kS) = o.s;
            }
            // reverse step
            for (int x = slen - 1; x >= 0; --x) {
                const long row = chain * T + t0 + s0 + x;
                Tok<D, M> tk;
                load_tok<D, M, true>(tk, A, row, col0);
                float Pp[D], Pq[D], Mp[CPL][D], e[CPL], u[D];
#pragma unroll
                for (int j = 0; j < D; ++j) Pp[j] = hx(x, H::kP + j);
#pragma unroll
                for (int l = 0; l < CPL; ++l) {
                    e[l] = hx(x, H::kE + l);
#pragma unroll
                    for (int i = 0; i < D; ++i) Mp[l][i] = hx(x, H::kM + l * D + i);
                }
                g.gather(hx(x, H::kU), u);
                const float beta = hx(x, H::kB), s = hx(x, H::kS);
#pragma unroll
                for (int j = 0; j < D; ++j) Pq[j] = g.xor_(Pp[j], 1);
                float bd[D], bo[D];
                a_rows(tk, bd, bo, false);
                float pbar[D];
                congruence_row<D>(Pp, Pq, pick(bd, own), pick(bo, own), bd, bo, pbar);
                add_pair_noise(pbar, tk.qp, own);
                const float u_own = pick(u, own), k_own = pick(tk.k, own);
                // mean side, lane's columns: M_bar, M_n, gM_n, ge
                float mbar[CPL][D], gmn[CPL][D], ge[CPL];
#pragma unroll
                for (int l = 0; l < CPL; ++l) {
#pragma unroll
                    for (int i = 0; i < D; ++i) {
                        mbar[l][i] = fmaf(bd[i], Mp[l][i], bo[i] * Mp[l][i ^ 1]);
                        gmn[l][i] = fmaf(tk.q[i], tk.gy[l], gM[l][i]);
                    }
                    float z = 0.f;
#pragma unroll
                    for (int i = 0; i < D; ++i) z = fmaf(gmn[l][i], u[i], z);
                    ge[l] = beta * z;
                }
                // per-row partial sums over the lane's columns: gq, h, M_bar ge,
                // and the mean parts of gA (i, i) and (i, i ^ 1)
                float parts[5][D];
#pragma unroll
                for (int i = 0; i < D; ++i) {
                    float zq = 0.f, zh = 0.f, zm = 0.f, zd = 0.f, zo = 0.f;
#pragma unroll
                    for (int l = 0; l < CPL; ++l) {
                        const float mn = fmaf(beta * u[i], e[l], mbar[l][i]);
                        zq = fmaf(mn, tk.gy[l], zq);
                        zh = fmaf(gmn[l][i], e[l], zh);
                        zm = fmaf(mbar[l][i], ge[l], zm);
                        const float gmb = fmaf(-tk.k[i], ge[l], gmn[l][i]);
                        zd = fmaf(gmb, Mp[l][i], zd);
                        zo = fmaf(gmb, Mp[l][i ^ 1], zo);
                    }
                    parts[0][i] = zq;
                    parts[1][i] = zh;
                    parts[2][i] = zm;
                    parts[3][i] = zd;
                    parts[4][i] = zo;
                }
                float tot[5];
                g.template reduce_scatter<5>(parts, tot);  // lane `own` gets row own
                const float gq_own = tot[0], h_own = tot[1], mge_own = tot[2];
                float ru = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) ru = fmaf(R[j], u[j], ru);
                const float gbeta = g.allsum(u_own * h_own - u_own * ru);
                const float gs = (s >= A.floor) ? -beta * beta * gbeta : 0.f;
                const float gu_own = fmaf(gs, k_own, beta * h_own - 2.f * beta * ru);
                float gu[D];
                g.gather(gu_own, gu);
                float pg = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) pg = fmaf(pbar[j], gu[j], pg);
                const float gk_own = pg + gs * u_own - mge_own;
                // S row own, symmetric; the partner's row for the congruences
                float S[D];
#pragma unroll
                for (int j = 0; j < D; ++j)
                    S[j] = R[j] + 0.5f * (__fmul_rn(gu_own, tk.k[j]) + __fmul_rn(gu[j], k_own));
                float Sq[D];
#pragma unroll
                for (int j = 0; j < D; ++j) Sq[j] = g.xor_(S[j], 1);
                // gA (i, k) = 2 sum_j S_ij (A Pp)_jk + mean part, k in {own, own ^ 1};
                // (A Pp)_jk = A_jj Pp_kj + A_j,j^1 Pp_k,j^1 (Pp symmetric)
                float ga_d = 0.f, ga_o = 0.f;
#pragma unroll
                for (int j = 0; j < D; ++j) {
                    const float apd = fmaf(bd[j], Pp[j], bo[j] * Pp[j ^ 1]);
                    const float apo = fmaf(bd[j], Pq[j], bo[j] * Pq[j ^ 1]);
                    ga_d = fmaf(S[j], apd, ga_d);
                    ga_o = fmaf(S[j], apo, ga_o);
                }
                ga_d = fmaf(2.f, ga_d, tot[3]);
                ga_o = fmaf(2.f, ga_o, tot[4]);
                // block m: g_c = gA(2m,2m) + gA(2m+1,2m+1); g_s = gA(2m+1,2m) - gA(2m,2m+1)
                const float pd = g.xor_(ga_d, 1), po = g.xor_(ga_o, 1);
                if ((own & 1) == 0) {
                    const int m = own >> 1;
                    A.gcos[row * J + m] = ga_d + pd;
                    A.gsin[row * J + m] = po - ga_o;
                    A.gproc[row * J + m] = pick(S, own);
                }
                A.gk[row * D + own] = gk_own;
                A.gq[row * D + own] = gq_own;
#pragma unroll
                for (int l = 0; l < CPL; ++l) A.gv[row * M + col0 + l] = ge[l];
                if (own == 0) A.gobs[row] = gs;
                // previous-token adjoint: gM <- A^T (gM_n - k ge^T), R <- A^T S A
#pragma unroll
                for (int l = 0; l < CPL; ++l) {
                    float gmb[D];
#pragma unroll
                    for (int i = 0; i < D; ++i) gmb[i] = fmaf(-tk.k[i], ge[l], gmn[l][i]);
#pragma unroll
                    for (int i = 0; i < D; ++i) gM[l][i] = fmaf(bd[i], gmb[i], -bo[i] * gmb[i ^ 1]);
                }
                float bdt[D], bot[D];
                a_rows(tk, bdt, bot, true);
                congruence_row<D>(S, Sq, pick(bdt, own), pick(bot, own), bdt, bot, R);
                (void)pown;
            }
        }
    }
    if constexpr (NEED_INIT) {
#pragma unroll
        for (int i = 0; i < D; ++i)
#pragma unroll
            for (int l = 0; l < CPL; ++l) A.gm0[chain * D * M + i * M + col0 + l] = gM[l][i];
#pragma unroll
        for (int j = 0; j < D; ++j) A.gc0[chain * D * D + own * D + j] = R[j];
    }
}

template <int D>
int launch(bool backward, bool init, const Args &a, cudaStream_t st) {
    const long blocks = (a.n * D + kThreads - 1) / kThreads;
    if (blocks > 0x7fffffffL) return fail(BSSM_ERR_INVALID, "rotation: too many chains");
    if (!backward) {
        rot_forward<D, 8><<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(a);
        return check_launch("rotation forward");
    }
    if (init) {
        rot_backward<D, 8, true><<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(a);
    } else {
        rot_backward<D, 8, false><<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(a);
    }
    return check_launch("rotation backward");
}

inline size_t workspace(int d, long n, long t, int chunks) {
    if (n <= 0 || t <= 0 || chunks <= 0) return 0;
    const long span = chunks < t ? chunks : t;
    const long nsub = (span + kSub - 1) / kSub;
    if (nsub <= 1) return 0;
    return static_cast<size_t>(n) * static_cast<size_t>(nsub - 1) * static_cast<size_t>(d) * (d + 8) * sizeof(float);
}

int run(int d, bool backward, bool init, const Args &a, cudaStream_t st) {
    switch (d) {
        case 2: return launch<2>(backward, init, a, st);
        case 4: return launch<4>(backward, init, a, st);
        case 8: return launch<8>(backward, init, a, st);
    }
    return fail(BSSM_ERR_UNSUPPORTED, "rotation dynamics: key_dim %d (supported: 2, 4, 8 with value_dim 8)", d);
}

}  // namespace rot
}  // namespace bssm

using bssm::fail;

extern "C" size_t bssm_rotation_workspace_bytes(int key_dim, int value_dim, long n, long t, int chunks) {
    if (value_dim != 8 || (key_dim != 2 && key_dim != 4 && key_dim != 8)) return 0;
    return bssm::rot::workspace(key_dim, n, t, chunks);
}

static int rotation_common(int d, int m, long n, long t, int chunks, double floor_) {
    if (m != 8 || (d != 2 && d != 4 && d != 8))
        return fail(BSSM_ERR_UNSUPPORTED, "rotation dynamics: (key_dim, value_dim) = (%d, %d); supported: "
                    "(2,8), (4,8), (8,8)", d, m);
    if (n < 0 || t < 0) return fail(BSSM_ERR_INVALID, "negative size n=%ld t=%ld", n, t);
    if (chunks <= 0) return fail(BSSM_ERR_INVALID, "chunks must be positive (got %d)", chunks);
    if (!(floor_ > 0.0) || floor_ != floor_ || floor_ > 3.0e38)
        return fail(BSSM_ERR_INVALID, "denominator_floor must be finite and positive");
    return BSSM_OK;
}

extern "C" int bssm_rotation_forward_chunked(int key_dim, int value_dim, const float *keys, const float *values,
                                             const float *queries, const float *cosines, const float *sines,
                                             const float *process, const float *observation, const float *mean0,
                                             const float *cov0, float *out, float *mean_final, float *cov_final,
                                             float *boundary_mean, float *boundary_cov, long n, long t, int chunks,
                                             double denominator_floor, void *stream) {
    int rc = rotation_common(key_dim, value_dim, n, t, chunks, denominator_floor);
    if (rc) return rc;
    if (n == 0) return BSSM_OK;
    if (!mean_final || !cov_final || !boundary_mean || !boundary_cov ||
        (t > 0 && (!keys || !values || !queries || !cosines || !sines || !process || !observation || !out)))
        return fail(BSSM_ERR_INVALID, "rotation forward: null pointer");
    bssm::rot::Args a{};
    a.keys = keys;
    a.values = values;
    a.queries = queries;
    a.cosines = cosines;
    a.sines = sines;
    a.process = process;
    a.observation = observation;
    a.mean0 = mean0;
    a.cov0 = cov0;
    a.out = out;
    a.mean_final = mean_final;
    a.cov_final = cov_final;
    a.bmean = boundary_mean;
    a.bcov = boundary_cov;
    a.n = n;
    a.t = t;
    a.chunks = chunks;
    a.floor = static_cast<float>(denominator_floor);
    return bssm::rot::run(key_dim, false, false, a, static_cast<cudaStream_t>(stream));
}

extern "C" int bssm_rotation_backward_chunked(
    int key_dim, int value_dim, int need_initial, const float *keys, const float *values, const float *queries,
    const float *cosines, const float *sines, const float *process, const float *observation,
    const float *boundary_mean, const float *boundary_cov, const float *grad_out, const float *grad_mean_final,
    const float *grad_cov_final, float *grad_keys, float *grad_values, float *grad_queries, float *grad_cosines,
    float *grad_sines, float *grad_process, float *grad_observation, float *grad_mean0, float *grad_cov0,
    void *workspace, size_t workspace_bytes, long n, long t, int chunks, double denominator_floor, void *stream) {
    int rc = rotation_common(key_dim, value_dim, n, t, chunks, denominator_floor);
    if (rc) return rc;
    if (n == 0) return BSSM_OK;
    const bool init = need_initial != 0;
    if (init && (!grad_mean0 || !grad_cov0))
        return fail(BSSM_ERR_INVALID, "rotation backward: need_initial requires grad_mean0/grad_cov0");
    if (!boundary_mean || !boundary_cov ||
        (t > 0 && (!keys || !values || !queries || !cosines || !sines || !process || !observation || !grad_keys ||
                   !grad_values || !grad_queries || !grad_cosines || !grad_sines || !grad_process ||
                   !grad_observation)))
        return fail(BSSM_ERR_INVALID, "rotation backward: null pointer");
    const size_t need = bssm::rot::workspace(key_dim, n, t, chunks);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return fail(BSSM_ERR_WORKSPACE, "rotation backward: workspace of %zu bytes required (got %zu)", need,
                    workspace_bytes);
    bssm::rot::Args a{};
    a.keys = keys;
    a.values = values;
    a.queries = queries;
    a.cosines = cosines;
    a.sines = sines;
    a.process = process;
    a.observation = observation;
    a.bmean = const_cast<float *>(boundary_mean);
    a.bcov = const_cast<float *>(boundary_cov);
    a.gy = grad_out;
    a.gmf = grad_mean_final;
    a.gcf = grad_cov_final;
    a.gk = grad_keys;
    a.gv = grad_values;
    a.gq = grad_queries;
    a.gcos = grad_cosines;
    a.gsin = grad_sines;
    a.gproc = grad_process;
    a.gobs = grad_observation;
    a.gm0 = grad_mean0;
    a.gc0 = grad_cov0;
    a.ws = static_cast<float *>(workspace);
    a.n = n;
    a.t = t;
    a.chunks = chunks;
    a.floor = static_cast<float>(denominator_floor);
    if (t == 0 && !init) return BSSM_OK;
    return bssm::rot::run(key_dim, true, init, a, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// The rotation coefficients rho cos(theta), rho sin(theta) from the caller's
// radii and angles, with the reference's radius handling (bayesian_layer.py:
// the radii clamped below at the smallest normal float and above at 1, then
// make_rotation_dynamics' exp(log(radius)) clipped at 1), and their backward
// as the chain of those operations' derivatives.  One pass over the elements
// each way instead of one per operation.  Products and the division are
// rounded separately (no contraction), as the separate operations round them.
// ---------------------------------------------------------------------------
namespace bssm {
namespace rot {

constexpr float kTinyRadius = 1.17549435e-38f;  // smallest normal float (torch.finfo(float32).tiny)

__device__ __forceinline__ void radius_chain(float r, float &t2, float &raw, float &rho) {
    const float t1 = r < kTinyRadius ? kTinyRadius : r;  // clamp_min (NaN passes through)
    t2 = t1 <= 1.0f ? t1 : 1.0f;
    raw = expf(logf(t2));
    rho = raw <= 1.0f ? raw : 1.0f;
}

__global__ void __launch_bounds__(256) coeff_kernel(const float *__restrict__ radii, const float *__restrict__ angles,
                                                    long count, float *__restrict__ cosines,
                                                    float *__restrict__ sines) {
    for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        float t2, raw, rho;
        radius_chain(__ldg(radii + i), t2, raw, rho);
        const float th = __ldg(angles + i);
        cosines[i] = __fmul_rn(rho, cosf(th));
        sines[i] = __fmul_rn(rho, sinf(th));
    }
}

__global__ void __launch_bounds__(256) coeff_backward_kernel(const float *__restrict__ radii,
                                                             const float *__restrict__ angles,
                                                             const float *__restrict__ gcos,
                                                             const float *__restrict__ gsin, long count,
                                                             float *__restrict__ gradii,
                                                             float *__restrict__ gangles) {
    for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
        const float r = __ldg(radii + i), th = __ldg(angles + i);
        float t2, raw, rho;
        radius_chain(r, t2, raw, rho);
        const float gc = gcos ? __ldg(gcos + i) : 0.f, gs = gsin ? __ldg(gsin + i) : 0.f;
        const float c = cosf(th), sn = sinf(th);
        // c_out = rho * cos(theta), s_out = rho * sin(theta)
        const float g_rho = __fadd_rn(__fmul_rn(gc, c), __fmul_rn(gs, sn));
        gangles[i] = __fadd_rn(__fmul_rn(__fmul_rn(gc, rho), -sn), __fmul_rn(__fmul_rn(gs, rho), c));
        const float g_raw = raw <= 1.0f ? g_rho : 0.f;          // rho = where(raw <= 1, raw, 1)
        const float g_log = __fmul_rn(g_raw, raw);              // raw = exp(l)
        const float g_t2 = __fdiv_rn(g_log, t2);                // l = log(t2)
        const float t1 = r < kTinyRadius ? kTinyRadius : r;
        const float g_t1 = t1 <= 1.0f ? g_t2 : 0.f;             // t2 = where(t1 <= 1, t1, 1)
        gradii[i] = r >= kTinyRadius ? g_t1 : 0.f;              // t1 = clamp_min(r, tiny)
    }
}

int coeff_grid(long count) {
    const long blocks = (count + 255) / 256;
    return static_cast<int>(blocks < 148L * 16 ? (blocks > 0 ? blocks : 1) : 148L * 16);
}

}  // namespace rot
}  // namespace bssm

extern "C" int bssm_rotation_coefficients(const float *radii, const float *angles, long count, float *cosines,
                                          float *sines, void *stream) {
    using namespace bssm;
    if (count < 0) return fail(BSSM_ERR_INVALID, "rotation coefficients: negative count");
    if (count == 0) {
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!radii || !angles || !cosines || !sines) return fail(BSSM_ERR_INVALID, "rotation coefficients: null pointer");
    rot::coeff_kernel<<<rot::coeff_grid(count), 256, 0, static_cast<cudaStream_t>(stream)>>>(radii, angles, count,
                                                                                            cosines, sines);
    return check_launch("rotation coefficients");
}

extern "C" int bssm_rotation_coefficients_backward(const float *radii, const float *angles, const float *grad_cosines,
                                                   const float *grad_sines, long count, float *grad_radii,
                                                   float *grad_angles, void *stream) {
    using namespace bssm;
    if (count < 0) return fail(BSSM_ERR_INVALID, "rotation coefficients backward: negative count");
    if (count == 0) {
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!radii || !angles || !grad_radii || !grad_angles)
        return fail(BSSM_ERR_INVALID, "rotation coefficients backward: null pointer");
    rot::coeff_backward_kernel<<<rot::coeff_grid(count), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        radii, angles, grad_cosines, grad_sines, count, grad_radii, grad_angles);
    return check_launch("rotation coefficients backward");
}

