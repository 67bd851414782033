// bssm_staged.cu -- shared-memory-staged chunked forward and replay backward.
//
// Same recurrence and adjoint as bssm_recurrence.cu (catid/bayes-ssm
// bayes_ssm/bayesian_layer.py:153-181, :207-251), reorganised for occupancy
// and latency hiding on sm_100a:
//
// * One warp per CTA serving C = 32/LPC chains; a chain is served by LPC
//   lanes, lane `sub` owning covariance rows sub*RPL.. (RPL = D/LPC) and mean
//   columns sub*CPL.. (CPL = M/LPC).
// * Token inputs arrive in shared memory as tiles of kS tokens x C chains,
//   copied with cp.async by all lanes, several tiles in flight; the compute
//   lanes never wait on a global load inside the recurrence.
// * Backward: per chunk (last to first) phase A replays the chunk from its
//   boundary checkpoint and saves the state at every kS-token boundary into
//   the workspace; phase B then, per kS-token sub-chunk (last to first),
//   replays the sub-chunk into a shared-memory history and runs the reverse
//   step over it.  The post-update mean of a sub-chunk's last token is the
//   replay's final state, so nothing is carried between sub-chunks except the
//   adjoints (dL/dM columns and R = sym(dL/dP) rows).
#include <cstdint>

#include "bayes_ssm_b200.h"
#include "bssm_common.cuh"
#include "bssm_internal.h"

namespace bssm {
namespace staged {

constexpr int kS = 4;          // tokens per tile = history sub-chunk
constexpr int kStagesFwd = 3;  // forward: tiles in flight
constexpr int kStagesBwd = 2;  // backward: one tile is consumed over a replay and a reverse pass

constexpr int al16(int x) { return (x + 15) / 16 * 16; }

// Bank check for one tile region: C chains of LPC lanes; chain c's data starts
// at byte c*cs.  Two access patterns are checked: every lane reading its own
// `lane_bytes`-wide slice (lane_bytes 0: all lanes of a chain read the same
// word), and the chain's lanes reading one shared 16-byte chunk.  Shared
// memory serves 128 bytes of distinct lanes per wavefront; within a wavefront
// two different words in the same bank conflict.
constexpr bool region_conflict_free(int cs, int lane_bytes, int C, int LPC) {
    const int patterns[2] = {lane_bytes, 16};
    for (int pi = 0; pi < 2; ++pi) {
        const int w = patterns[pi];
        const bool bcast = (w == 0 || w == 16);  // one address per chain
        const int access = (w == 0) ? 4 : w;
        const int lanes_per_wave = 128 / access < 32 ? 128 / access : 32;
        const int chains_per_wave = lanes_per_wave / LPC > 0 ? lanes_per_wave / LPC : 1;
        for (int c0 = 0; c0 < C; c0 += chains_per_wave) {
            int owner[32] = {};
            for (int b = 0; b < 32; ++b) owner[b] = -1;
            for (int c = c0; c < c0 + chains_per_wave && c < C; ++c) {
                for (int sub = 0; sub < (bcast ? 1 : LPC); ++sub) {
                    const int word0 = (c * cs + (bcast ? 0 : sub * access)) / 4;
                    for (int x = 0; x < access / 4; ++x) {
                        const int word = word0 + x, bank = word % 32;
                        if (owner[bank] >= 0 && owner[bank] != word) return false;
                        owner[bank] = word;
                    }
                }
            }
        }
    }
    return true;
}
// Smallest 16-byte-padded chain stride >= bytes that is conflict free.
constexpr int chain_stride(int bytes, int lane_bytes, int C, int LPC) {
    for (int pad = 0; pad <= 128; pad += 16)
        if (region_conflict_free(al16(bytes) + pad, lane_bytes, C, LPC)) return al16(bytes) + pad;
    return al16(bytes);
}

template <int D, int M, int LPC, typename TIn>
struct Geo {
    static constexpr int RPL = D / LPC, CPL = M / LPC, C = 32 / LPC;
    static_assert(D % LPC == 0 && M % LPC == 0, "lanes per chain must divide D and M");
    // tile (bytes)
    static constexpr int rbK = D * static_cast<int>(sizeof(TIn)), rbV = M * static_cast<int>(sizeof(TIn));
    static constexpr int rbA = D * 4, rbG = M * 4, rbP = 4;
    // each lane reads its own RPL keys / decays and CPL values / gy entries
    static constexpr int csK = chain_stride(kS * rbK, RPL * static_cast<int>(sizeof(TIn)), C, LPC);
    static constexpr int csV = chain_stride(kS * rbV, CPL * static_cast<int>(sizeof(TIn)), C, LPC);
    static constexpr int csA = chain_stride(kS * rbA, RPL * 4, C, LPC);
    static constexpr int csG = chain_stride(kS * rbG, CPL * 4, C, LPC);
    static constexpr int csP = chain_stride(kS * rbP, 0, C, LPC);
    static constexpr int oK = 0, oQ = oK + C * csK, oV = oQ + C * csK, oA = oV + C * csV;
    static constexpr int oG = oA + C * csA, oP = oG + C * csG, oR = oP + C * csP, kTile = oR + C * csP;
    // history (floats).  Per chain, the lane-private blocks of the pre-token
    // mean and covariance: [token][lane-interleaved 4-float chunks], chain
    // stride == 16 (mod 32) so the two chains of a 128-bit wavefront use
    // different banks.  Then, shared by the CTA and indexed [token][chain][.],
    // the small vectors u (D), e (M) and (beta, s).
    static constexpr int hMB = CPL * D, hPB = RPL * D;  // lane blocks per token
    static constexpr int hM = 0, hP = hM + kS * M * D, kMPRaw = hP + kS * D * D;
    static constexpr int kHistMP = kMPRaw + ((16 - kMPRaw % 32) + 32) % 32;
    static constexpr int hU = C * kHistMP, hE = hU + kS * C * D, hB = hE + kS * C * M;
    static constexpr int kHistAll = hB + kS * C * 2;
    // phase-A workspace (floats per chain per saved state)
    static constexpr int kWsLane = (hMB + hPB + 3) / 4 * 4, kWsChain = kWsLane * LPC;
};

// Lane-private history block of B floats: 4-float chunks interleaved across
// the group's lanes so that a group's 128-bit accesses hit distinct banks.
template <int B, int LPC>
__device__ __forceinline__ float *lane_block(float *base, int sub, int x) {
    if constexpr (B >= 4) {
        return base + (x * LPC + sub) * 4;
    } else {
        return base + sub * B;
    }
}
template <int B, int LPC>
__device__ __forceinline__ void put_block(float *base, int sub, const float (&v)[B]) {
    if constexpr (B >= 4) {
#pragma unroll
        for (int x = 0; x < B / 4; ++x)
            *reinterpret_cast<float4 *>(lane_block<B, LPC>(base, sub, x)) =
                make_float4(v[4 * x], v[4 * x + 1], v[4 * x + 2], v[4 * x + 3]);
    } else {
        sts_vec<B>(base + sub * B, v);
    }
}
template <int B, int LPC>
__device__ __forceinline__ void get_block(const float *base, int sub, float (&v)[B]) {
    if constexpr (B >= 4) {
#pragma unroll
        for (int x = 0; x < B / 4; ++x) {
            const float4 w = *reinterpret_cast<const float4 *>(lane_block<B, LPC>(const_cast<float *>(base), sub, x));
            v[4 * x] = w.x; v[4 * x + 1] = w.y; v[4 * x + 2] = w.z; v[4 * x + 3] = w.w;
        }
    } else {
        lds_vec<B>(base + sub * B, v);
    }
}

// Copy rows [t0, t0+ntok) of chains [n0, n0+nvalid) of a [N,T,RB-byte] tensor
// into a tile region (chain stride CS bytes), split over the warp's lanes.
template <int RB, int CS, int C>
__device__ __forceinline__ void issue_rows(uint32_t sdst, const void *gbase, long T, long n0, int nvalid,
                                           long t0, int ntok, int lane) {
    constexpr int G = RB >= 16 ? 16 : RB;
    static_assert(G >= 4 && RB % G == 0, "row bytes");
    constexpr int PPR = RB / G;
    constexpr int TOTAL = C * kS * PPR;
    const char *g = static_cast<const char *>(gbase);
#pragma unroll
    for (int it = 0; it < (TOTAL + 31) / 32; ++it) {
        const int p = lane + it * 32;
        if (TOTAL % 32 == 0 || p < TOTAL) {
            const int c = p / (kS * PPR);
            const int rem = p - c * (kS * PPR);
            const int tau = rem / PPR;
            const int part = rem - tau * PPR;
            if (c < nvalid && tau < ntok) {
                const char *src = g + ((n0 + c) * T + t0 + tau) * RB + part * G;
                cp_async<G>(sdst + c * CS + tau * RB + part * G, src);
            }
        }
    }
}

enum TileKind { kForward = 0, kPhaseA = 1, kPhaseB = 2 };

template <int D, int M, int LPC, bool FIXED, typename TIn>
struct Inputs {
    const TIn *keys, *values, *queries;
    const float *decay, *process, *observation, *gy;
};

template <int D, int M, int LPC, bool FIXED, typename TIn>
__device__ __forceinline__ void issue_tile(char *stage, const Inputs<D, M, LPC, FIXED, TIn> &in, int kind,
                                           long T, long n0, int nvalid, long t0, int ntok, int lane) {
    using G = Geo<D, M, LPC, TIn>;
    const uint32_t s = smem_u32(stage);
    issue_rows<G::rbK, G::csK, G::C>(s + G::oK, in.keys, T, n0, nvalid, t0, ntok, lane);
    issue_rows<G::rbV, G::csV, G::C>(s + G::oV, in.values, T, n0, nvalid, t0, ntok, lane);
    if (kind != kPhaseA) issue_rows<G::rbK, G::csK, G::C>(s + G::oQ, in.queries, T, n0, nvalid, t0, ntok, lane);
    if constexpr (!FIXED) {
        issue_rows<G::rbA, G::csA, G::C>(s + G::oA, in.decay, T, n0, nvalid, t0, ntok, lane);
        issue_rows<G::rbP, G::csP, G::C>(s + G::oP, in.process, T, n0, nvalid, t0, ntok, lane);
        issue_rows<G::rbP, G::csP, G::C>(s + G::oR, in.observation, T, n0, nvalid, t0, ntok, lane);
    }
    if (kind == kPhaseB && in.gy != nullptr)
        issue_rows<G::rbG, G::csG, G::C>(s + G::oG, in.gy, T, n0, nvalid, t0, ntok, lane);
}

// Ask L2 to start fetching a saved state (mean + covariance, `floats` floats)
// that this chain will load at its next sub-chunk; the lanes split the lines.
template <int LPC>
__device__ __forceinline__ void prefetch_state_l2(const float *p, int floats, int sub) {
    const int lines = (floats * 4 + 127) / 128;
    for (int l = sub; l < lines; l += LPC)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(p + l * 32));
}

// ---------------------------------------------------------------------------
// Lane-relative row order.
//
// Lane `sub` owns rows sub*RPL .. sub*RPL+RPL-1.  It keeps every row-indexed
// vector -- keys, decays, queries, gains, its mean columns, the columns of its
// covariance rows and the matching adjoints -- in the order
//     position x  <->  row x ^ (sub*RPL).
// Its own rows then sit at the fixed positions 0 .. RPL-1 (so the diagonal of
// its covariance rows is at a compile-time position), and the reduce-scatter
// of per-row partial sums needs no selects (LaneGroup::reduce_scatter_lane).
// Global and shared-memory copies of the state stay in plain row order; the
// helpers below translate.
// ---------------------------------------------------------------------------
template <int D, int LPC>
__device__ __forceinline__ int lane_row(int x, int sub) { return x ^ (sub * (D / LPC)); }

// D row-indexed elements at `base` (plain order) -> lane order.
template <int D, int LPC, typename T>
__device__ __forceinline__ void lds_rows(const T *base, int sub, float (&out)[D]) {
    constexpr int RPL = D / LPC;
#pragma unroll
    for (int m = 0; m < LPC; ++m) {
        float chunk[RPL];
        lds_vec<RPL>(base + (m ^ sub) * RPL, chunk);
#pragma unroll
        for (int i = 0; i < RPL; ++i) out[m * RPL + i] = chunk[i];
    }
}
// Global row (D floats, plain order) <-> lane order.
template <int D, int LPC>
__device__ __forceinline__ void ldg_row(const float *rowp, int sub, float (&out)[D]) {
    constexpr int RPL = D / LPC;
#pragma unroll
    for (int m = 0; m < LPC; ++m) {
        float chunk[RPL];
        load_vec<RPL>(rowp + (m ^ sub) * RPL, chunk);
#pragma unroll
        for (int i = 0; i < RPL; ++i) out[m * RPL + i] = chunk[i];
    }
}
template <int D, int LPC>
__device__ __forceinline__ void stg_row(float *rowp, int sub, const float (&v)[D]) {
    constexpr int RPL = D / LPC;
#pragma unroll
    for (int m = 0; m < LPC; ++m) {
        float chunk[RPL];
#pragma unroll
        for (int i = 0; i < RPL; ++i) chunk[i] = v[m * RPL + i];
        store_vec<RPL>(rowp + (m ^ sub) * RPL, chunk);
    }
}
// The lane's CPL columns (col0 ..) of a row-major [D, M] mean, rows in lane order.
template <int D, int M, int LPC>
__device__ __forceinline__ void ldg_mean_cols(const float *base, int col0, int sub, float (&Mc)[M / LPC][D]) {
    constexpr int CPL = M / LPC;
#pragma unroll
    for (int x = 0; x < D; ++x) {
        float row[CPL];
        load_vec<CPL>(base + lane_row<D, LPC>(x, sub) * M + col0, row);
#pragma unroll
        for (int l = 0; l < CPL; ++l) Mc[l][x] = row[l];
    }
}
template <int D, int M, int LPC>
__device__ __forceinline__ void stg_mean_cols(float *base, int col0, int sub, const float (&Mc)[M / LPC][D]) {
    constexpr int CPL = M / LPC;
#pragma unroll
    for (int x = 0; x < D; ++x) {
        float row[CPL];
#pragma unroll
        for (int l = 0; l < CPL; ++l) row[l] = Mc[l][x];
        store_vec<CPL>(base + lane_row<D, LPC>(x, sub) * M + col0, row);
    }
}

// One token's inputs for this lane, read from a staged tile (keys and decays
// in lane order: the lane's own rows at positions 0 .. RPL-1).
template <int D, int M, int LPC>
struct Tok {
    float k[D], a[D], v[M / LPC];
    float p, r;
};

template <int D, int M, int LPC, bool FIXED, typename TIn>
__device__ __forceinline__ void read_tok(const char *stage, int c, int tau, int sub, Tok<D, M, LPC> &tk) {
    using G = Geo<D, M, LPC, TIn>;
    constexpr int CPL = G::CPL;
    lds_rows<D, LPC>(reinterpret_cast<const TIn *>(stage + G::oK + c * G::csK + tau * G::rbK), sub, tk.k);
    lds_vec<CPL>(reinterpret_cast<const TIn *>(stage + G::oV + c * G::csV + tau * G::rbV) + sub * CPL, tk.v);
    if constexpr (FIXED) {
#pragma unroll
        for (int j = 0; j < D; ++j) tk.a[j] = kFixedDecay;
        tk.p = kFixedProcess;
        tk.r = kFixedObservation;
    } else {
        lds_rows<D, LPC>(reinterpret_cast<const float *>(stage + G::oA + c * G::csA + tau * G::rbA), sub, tk.a);
        tk.p = reinterpret_cast<const float *>(stage + G::oP + c * G::csP)[tau];
        tk.r = reinterpret_cast<const float *>(stage + G::oR + c * G::csP)[tau];
    }
}

// One predict/update step on the lane's slice (own rows, own columns), all
// row-indexed arrays in lane order.
template <int D, int M, int LPC>
__device__ __forceinline__ void forward_step(const LaneGroup<LPC> &g, const Tok<D, M, LPC> &tk, float floor_,
                                             float (&Mc)[M / LPC][D], float (&P)[D / LPC][D], float (&u)[D],
                                             float (&u_own)[D / LPC], float (&e)[M / LPC], float &beta,
                                             float &s) {
    constexpr int RPL = D / LPC, CPL = M / LPC;
    float wk[D];
#pragma unroll
    for (int x = 0; x < D; ++x) wk[x] = tk.a[x] * tk.k[x];
    float sp = 0.f;
#pragma unroll
    for (int r = 0; r < RPL; ++r) {
        float z = 0.f;
#pragma unroll
        for (int x = 0; x < D; ++x) z = fmaf(P[r][x], wk[x], z);
        u_own[r] = fmaf(tk.a[r], z, tk.p * tk.k[r]);
        sp = fmaf(tk.k[r], u_own[r], sp);
    }
#pragma unroll
    for (int l = 0; l < CPL; ++l) {
        float acc = 0.f;
#pragma unroll
        for (int x = 0; x < D; ++x) acc = fmaf(Mc[l][x], wk[x], acc);
        e[l] = tk.v[l] - acc;
    }
    g.template gather_lane<RPL>(u_own, u);
    // s = r + k.u as a butterfly sum: bit-identical in every lane of the chain
    s = tk.r + g.allsum(sp);
    beta = 1.0f / (s < floor_ ? floor_ : s);  // clamp_min: NaN stays NaN
#pragma unroll
    for (int l = 0; l < CPL; ++l) {
        const float be = beta * e[l];
#pragma unroll
        for (int x = 0; x < D; ++x) Mc[l][x] = fmaf(tk.a[x], Mc[l][x], be * u[x]);
    }
    // rows of P' = A P A + p I - beta u u^T from commutative products and a
    // chain-wide beta, so the rows of different lanes stay bit-for-bit
    // symmetric; the diagonal entry of own row r is at position r
#pragma unroll
    for (int r = 0; r < RPL; ++r) {
#pragma unroll
        for (int x = 0; x < D; ++x) {
            const float upd = fmaf(-beta, u_own[r] * u[x], (tk.a[r] * tk.a[x]) * P[r][x]);
            P[r][x] = (x == r) ? upd + tk.p : upd;
        }
    }
}

// Plain-order token inputs and step, used by the forward kernel: the own
// rows' values are separate loads and the diagonal update is a select.  For
// the latency-bound forward this measured faster than the lane-relative
// order, which trades them for more, narrower shared-memory loads.
template <int D, int M, int LPC>
struct TokPlain {
    float k[D], a[D], v[M / LPC];
    float p, r;
    float k_own[D / LPC], a_own[D / LPC];
};

template <int D, int M, int LPC, bool FIXED, typename TIn>
__device__ __forceinline__ void read_tok_plain(const char *stage, int c, int tau, int sub, TokPlain<D, M, LPC> &tk) {
    using G = Geo<D, M, LPC, TIn>;
    constexpr int RPL = G::RPL, CPL = G::CPL;
    const TIn *kr = reinterpret_cast<const TIn *>(stage + G::oK + c * G::csK + tau * G::rbK);
    lds_vec<D>(kr, tk.k);
    lds_vec<CPL>(reinterpret_cast<const TIn *>(stage + G::oV + c * G::csV + tau * G::rbV) + sub * CPL, tk.v);
    if constexpr (FIXED) {
#pragma unroll
        for (int j = 0; j < D; ++j) tk.a[j] = kFixedDecay;
        tk.p = kFixedProcess;
        tk.r = kFixedObservation;
#pragma unroll
        for (int r = 0; r < RPL; ++r) tk.a_own[r] = kFixedDecay;
    } else {
        const float *ar = reinterpret_cast<const float *>(stage + G::oA + c * G::csA + tau * G::rbA);
        lds_vec<D>(ar, tk.a);
        lds_vec<RPL>(ar + sub * RPL, tk.a_own);
        tk.p = reinterpret_cast<const float *>(stage + G::oP + c * G::csP)[tau];
        tk.r = reinterpret_cast<const float *>(stage + G::oR + c * G::csP)[tau];
    }
    lds_vec<RPL>(kr + sub * RPL, tk.k_own);
}

// One predict/update step on the lane's slice (rows row0.., columns col0..).
template <int D, int M, int LPC>
__device__ __forceinline__ void forward_step_plain(const LaneGroup<LPC> &g, const TokPlain<D, M, LPC> &tk, float floor_,
                                             float (&Mc)[M / LPC][D], float (&P)[D / LPC][D], float (&u)[D],
                                             float (&u_own)[D / LPC], float (&e)[M / LPC], float &beta,
                                             float &s) {
    constexpr int RPL = D / LPC, CPL = M / LPC;
    const int row0 = g.sub * RPL;
    float wk[D];
#pragma unroll
    for (int j = 0; j < D; ++j) wk[j] = tk.a[j] * tk.k[j];
#pragma unroll
    for (int r = 0; r < RPL; ++r) {
        float z = 0.f;
#pragma unroll
        for (int j = 0; j < D; ++j) z = fmaf(P[r][j], wk[j], z);
        u_own[r] = fmaf(tk.a_own[r], z, tk.p * tk.k_own[r]);
    }
#pragma unroll
    for (int l = 0; l < CPL; ++l) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < D; ++i) acc = fmaf(Mc[l][i], wk[i], acc);
        e[l] = tk.v[l] - acc;
    }
    g.template gather_rows<RPL>(u_own, u);
    s = tk.r;
#pragma unroll
    for (int j = 0; j < D; ++j) s = fmaf(tk.k[j], u[j], s);
    beta = 1.0f / (s < floor_ ? floor_ : s);  // clamp_min: NaN stays NaN
#pragma unroll
    for (int l = 0; l < CPL; ++l) {
        const float be = beta * e[l];
#pragma unroll
        for (int i = 0; i < D; ++i) Mc[l][i] = fmaf(tk.a[i], Mc[l][i], be * u[i]);
    }
    // rows of P' = A P A + p I - beta u u^T from commutative products only,
    // so the rows of different lanes stay bit-for-bit symmetric
#pragma unroll
    for (int r = 0; r < RPL; ++r) {
#pragma unroll
        for (int j = 0; j < D; ++j) {
            const float upd = fmaf(-beta, u_own[r] * u[j], (tk.a_own[r] * tk.a[j]) * P[r][j]);
            P[r][j] = (j == row0 + r) ? upd + tk.p : upd;
        }
    }
}

// ===========================================================================
// Forward
// ===========================================================================
template <int D, int M, int LPC, bool FIXED, typename TIn>
__global__ void __launch_bounds__(32) forward_staged(const FwdArgs<TIn> A) {
    using G = Geo<D, M, LPC, TIn>;
    constexpr int RPL = G::RPL, CPL = G::CPL, C = G::C;
    extern __shared__ __align__(128) char smem[];
    const LaneGroup<LPC> g;
    const int lane = threadIdx.x;
    const int c = lane / LPC;
    const long n0 = static_cast<long>(blockIdx.x) * C;
    const long chain = n0 + c;
    const bool active = chain < A.n;
    const int nvalid = static_cast<int>((A.n - n0) < C ? (A.n - n0) : C);
    const int sub = g.sub;
    const int row0 = sub * RPL, col0 = sub * CPL;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;
    const Inputs<D, M, LPC, FIXED, TIn> in{A.keys, A.values, A.queries, A.decay, A.process, A.observation, nullptr};

    float Mc[CPL][D], P[RPL][D];
#pragma unroll
    for (int l = 0; l < CPL; ++l)
#pragma unroll
        for (int i = 0; i < D; ++i) Mc[l][i] = 0.f;
#pragma unroll
    for (int r = 0; r < RPL; ++r)
#pragma unroll
        for (int j = 0; j < D; ++j) P[r][j] = (j == row0 + r) ? 1.f : 0.f;
    if (active && A.mean0 != nullptr) load_mean_cols_g<D, M, CPL>(A.mean0 + chain * D * M, col0, Mc);
    if (active && A.cov0 != nullptr) {
        const float *c0 = A.cov0 + chain * D * D;
#pragma unroll
        for (int r = 0; r < RPL; ++r)
#pragma unroll
            for (int j = 0; j < D; ++j) P[r][j] = 0.5f * (c0[(row0 + r) * D + j] + c0[j * D + row0 + r]);
    }
    float *bm = A.bmean + chain * (nb + 1) * D * M;
    float *bc = A.bcov + chain * (nb + 1) * D * D;

    const long ntile = (T + kS - 1) / kS;
#pragma unroll
    for (int s = 0; s < kStagesFwd - 1; ++s) {
        if (s < ntile)
            issue_tile<D, M, LPC, FIXED, TIn>(smem + s * G::kTile, in, kForward, T, n0, nvalid, s * kS,
                                              static_cast<int>((T - s * kS) < kS ? (T - s * kS) : kS), lane);
        cp_async_commit();
    }
    long ckpt = 0;
    const long rs_slots = replay_slots_per_chunk(T, L);
    for (long q = 0; q < ntile; ++q) {
        const long qn = q + kStagesFwd - 1;
        if (qn < ntile)
            issue_tile<D, M, LPC, FIXED, TIn>(smem + (qn % kStagesFwd) * G::kTile, in, kForward, T, n0, nvalid,
                                              qn * kS, static_cast<int>((T - qn * kS) < kS ? (T - qn * kS) : kS),
                                              lane);
        cp_async_commit();
        cp_async_wait<kStagesFwd - 1>();
        __syncwarp();
        const char *stage = smem + (q % kStagesFwd) * G::kTile;
        const long t0 = q * kS;
        const int ntok = static_cast<int>((T - t0) < kS ? (T - t0) : kS);
        for (int tau = 0; tau < ntok; ++tau) {
            const long t = t0 + tau;
            if (t == ckpt * L) {
                if (active) {
                    store_mean_cols_g<D, M, CPL>(bm + ckpt * D * M, col0, Mc);
#pragma unroll
                    for (int r = 0; r < RPL; ++r) store_vec<D>(bc + ckpt * D * D + (row0 + r) * D, P[r]);
                }
                ++ckpt;
            } else if (A.rs != nullptr && (t - (ckpt - 1) * L) % kReplaySpan == 0) {
                if (active) {
                    const long base = replay_state_base(chain, nb, rs_slots, ckpt - 1,
                                                        (t - (ckpt - 1) * L) / kReplaySpan,
                                                        replay_state_floats(D, M));
                    rs_put_mean_cols<D, M, CPL>(A.rs, base, col0, Mc);
#pragma unroll
                    for (int r = 0; r < RPL; ++r) rs_put_row<D, M>(A.rs, base, row0 + r, P[r]);
                }
            }
            TokPlain<D, M, LPC> tk;
            read_tok_plain<D, M, LPC, FIXED, TIn>(stage, c, tau, sub, tk);
            float u[D], u_own[RPL], e[CPL], beta, s;
            forward_step_plain<D, M, LPC>(g, tk, A.floor, Mc, P, u, u_own, e, beta, s);
            if (active && A.rs != nullptr) {
                float *const gu = replay_gains(A.rs, A.n, T, L, D, M) + (chain * T + t) * D + row0;
#pragma unroll
                for (int r = 0; r < RPL; ++r) gu[r] = u_own[r];
                if (sub == 0)
                    replay_gain_scales(A.rs, A.n, T, L, D, M)[chain * T + t] = signed_gain_scale(beta, s, A.floor);
            }
            float qv[D];
            lds_vec<D>(reinterpret_cast<const TIn *>(stage + G::oQ + c * G::csK + tau * G::rbK), qv);
            float y[CPL];
#pragma unroll
            for (int l = 0; l < CPL; ++l) {
                float acc = 0.f;
#pragma unroll
                for (int i = 0; i < D; ++i) acc = fmaf(Mc[l][i], qv[i], acc);
                y[l] = acc;
            }
            if (active) store_vec<CPL>(A.out + (chain * T + t) * M + col0, y);
        }
        __syncwarp();
    }
    cp_async_wait<0>();
    if (active) {
        store_mean_cols_g<D, M, CPL>(bm + nb * D * M, col0, Mc);
        store_mean_cols_g<D, M, CPL>(A.mean_final + chain * D * M, col0, Mc);
#pragma unroll
        for (int r = 0; r < RPL; ++r) {
            store_vec<D>(bc + nb * D * D + (row0 + r) * D, P[r]);
            store_vec<D>(A.cov_final + chain * D * D + (row0 + r) * D, P[r]);
        }
    }
}

// ===========================================================================
// Backward
// ===========================================================================

// Order in which tiles are consumed (and therefore requested): for each chunk
// from the last, phase A sub-chunks 0 .. nsub-2 then phase B sub-chunks
// nsub-1 .. 0.
struct Schedule {
    long ci;
    int phase, j, nsub, len;
    bool done, skipA;
    long T;
    int L;
    __device__ __forceinline__ void enter_chunk() {
        const long t0 = ci * L;
        len = static_cast<int>((T - t0) < L ? (T - t0) : L);
        nsub = (len + kS - 1) / kS;
        if (nsub > 1 && !skipA) {
            phase = kPhaseA;
            j = 0;
        } else {
            phase = kPhaseB;
            j = nsub - 1;
        }
    }
    __device__ __forceinline__ void init(long T_, int L_, bool skipA_) {
        T = T_;
        L = L_;
        skipA = skipA_;
        ci = (T + L - 1) / L - 1;
        done = ci < 0;
        if (!done) enter_chunk();
    }
    __device__ __forceinline__ void advance() {
        if (phase == kPhaseA) {
            if (++j > nsub - 2) {
                phase = kPhaseB;
                j = nsub - 1;
            }
        } else if (--j < 0) {
            if (--ci < 0) {
                done = true;
            } else {
                enter_chunk();
            }
        }
    }
    __device__ __forceinline__ long t0() const { return ci * L + static_cast<long>(j) * kS; }
    __device__ __forceinline__ int ntok() const { return (len - j * kS) < kS ? (len - j * kS) : kS; }
};

template <int D, int M, int LPC, bool FIXED, bool NEED_DYN, bool NEED_INIT, typename TIn>
__global__ void __launch_bounds__(32) backward_staged(const BwdArgs<TIn> A) {
    using G = Geo<D, M, LPC, TIn>;
    constexpr int RPL = G::RPL, CPL = G::CPL, C = G::C;
    extern __shared__ __align__(128) char smem[];
    const LaneGroup<LPC> g;
    const int lane = threadIdx.x;
    const int c = lane / LPC;
    const long n0 = static_cast<long>(blockIdx.x) * C;
    const long chain = n0 + c;
    const bool active = chain < A.n;
    const int nvalid = static_cast<int>((A.n - n0) < C ? (A.n - n0) : C);
    const int sub = g.sub;
    const int row0 = sub * RPL, col0 = sub * CPL;
    const long T = A.t;
    const int L = A.chunks;
    const long nb = (T + L - 1) / L;
    const int nsub_max = (static_cast<int>(L < T ? L : T) + kS - 1) / kS;
    const float floor_ = A.floor;
    const bool has_gy = A.gy != nullptr;
    const Inputs<D, M, LPC, FIXED, TIn> in{A.keys, A.values, A.queries, A.decay, A.process, A.observation, A.gy};
    float *const hist_all = reinterpret_cast<float *>(smem + kStagesBwd * G::kTile);
    float *const hist = hist_all + c * G::kHistMP;  // this chain's mean/covariance blocks
    auto hU_at = [&](int tau) { return hist_all + G::hU + (tau * C + c) * D; };
    auto hE_at = [&](int tau) { return hist_all + G::hE + (tau * C + c) * M; };
    auto hB_at = [&](int tau) { return hist_all + G::hB + (tau * C + c) * 2; };
    const float *bm = A.bmean + chain * (nb + 1) * D * M;
    const float *bc = A.bcov + chain * (nb + 1) * D * D;
    float *ws = A.ws + chain * static_cast<long>(nsub_max > 1 ? nsub_max - 1 : 0) * G::kWsChain + sub * G::kWsLane;
    constexpr long kWsChain = G::kWsChain;

    float gM[CPL][D], R[RPL][D];
#pragma unroll
    for (int l = 0; l < CPL; ++l)
#pragma unroll
        for (int i = 0; i < D; ++i) gM[l][i] = 0.f;
#pragma unroll
    for (int r = 0; r < RPL; ++r)
#pragma unroll
        for (int j = 0; j < D; ++j) R[r][j] = 0.f;
    if (active && A.gmf != nullptr) ldg_mean_cols<D, M, LPC>(A.gmf + chain * D * M, col0, sub, gM);
    if (active && A.gcf != nullptr) {
        const float *gc = A.gcf + chain * D * D;
#pragma unroll
        for (int r = 0; r < RPL; ++r)
#pragma unroll
            for (int x = 0; x < D; ++x) {
                const int j = lane_row<D, LPC>(x, sub);
                R[r][x] = 0.5f * (gc[(row0 + r) * D + j] + gc[j * D + row0 + r]);
            }
    }

    const bool have_rs = A.rs != nullptr;
    Schedule prod;
    prod.init(T, L, have_rs);
#pragma unroll
    for (int s = 0; s < kStagesBwd - 1; ++s) {
        if (!prod.done) {
            issue_tile<D, M, LPC, FIXED, TIn>(smem + s * G::kTile, in, prod.phase, T, n0, nvalid, prod.t0(),
                                              prod.ntok(), lane);
            prod.advance();
        }
        cp_async_commit();
    }
    long qc = 0;  // tiles consumed
    auto acquire = [&]() -> const char * {
        if (!prod.done) {
            issue_tile<D, M, LPC, FIXED, TIn>(smem + ((qc + kStagesBwd - 1) % kStagesBwd) * G::kTile, in, prod.phase,
                                              T, n0, nvalid, prod.t0(), prod.ntok(), lane);
            prod.advance();
        }
        cp_async_commit();
        cp_async_wait<kStagesBwd - 1>();
        __syncwarp();
        return smem + (qc % kStagesBwd) * G::kTile;
    };

    for (long ci = nb - 1; ci >= 0; --ci) {
        const long t0c = ci * L;
        const int len = static_cast<int>((T - t0c) < L ? (T - t0c) : L);
        const int nsub = (len + kS - 1) / kS;

        // ---- phase A (skipped when the forward saved the replay states)
        if (nsub > 1 && !have_rs) {
            float Mc[CPL][D], P[RPL][D];
            if (active) {
                ldg_mean_cols<D, M, LPC>(bm + ci * D * M, col0, sub, Mc);
#pragma unroll
                for (int r = 0; r < RPL; ++r) ldg_row<D, LPC>(bc + ci * D * D + (row0 + r) * D, sub, P[r]);
            } else {
#pragma unroll
                for (int l = 0; l < CPL; ++l)
#pragma unroll
                    for (int i = 0; i < D; ++i) Mc[l][i] = 0.f;
#pragma unroll
                for (int r = 0; r < RPL; ++r)
#pragma unroll
                    for (int x = 0; x < D; ++x) P[r][x] = (x == r) ? 1.f : 0.f;
            }
            for (int j = 0; j + 1 < nsub; ++j) {
                const char *stage = acquire();
#pragma unroll
                for (int tau = 0; tau < kS; ++tau) {
                    Tok<D, M, LPC> tk;
                    read_tok<D, M, LPC, FIXED, TIn>(stage, c, tau, sub, tk);
                    float u[D], u_own[RPL], e[CPL], beta, s;
                    forward_step<D, M, LPC>(g, tk, floor_, Mc, P, u, u_own, e, beta, s);
                }
                if (active) {
                    float flat[G::kWsLane];
#pragma unroll
                    for (int x = 0; x < G::kWsLane; ++x) flat[x] = 0.f;
#pragma unroll
                    for (int l = 0; l < CPL; ++l)
#pragma unroll
                        for (int i = 0; i < D; ++i) flat[l * D + i] = Mc[l][i];
#pragma unroll
                    for (int r = 0; r < RPL; ++r)
#pragma unroll
                        for (int jj = 0; jj < D; ++jj) flat[G::hMB + r * D + jj] = P[r][jj];
                    store_vec<G::kWsLane>(ws + j * kWsChain, flat);
                }
                __syncwarp();
                ++qc;
            }
        }

        // ---- phase B
        for (int j = nsub - 1; j >= 0; --j) {
            const char *stage = acquire();
            const int slen = (len - j * kS) < kS ? (len - j * kS) : kS;
            float Mc[CPL][D], P[RPL][D];
            if (!active) {
#pragma unroll
                for (int l = 0; l < CPL; ++l)
#pragma unroll
                    for (int i = 0; i < D; ++i) Mc[l][i] = 0.f;
#pragma unroll
                for (int r = 0; r < RPL; ++r)
#pragma unroll
                    for (int x = 0; x < D; ++x) P[r][x] = (x == r) ? 1.f : 0.f;
            } else if (j == 0) {
                ldg_mean_cols<D, M, LPC>(bm + ci * D * M, col0, sub, Mc);
#pragma unroll
                for (int r = 0; r < RPL; ++r) ldg_row<D, LPC>(bc + ci * D * D + (row0 + r) * D, sub, P[r]);
            } else if (have_rs) {
                const long base = replay_state_base(chain, nb, nsub_max - 1, ci, j, replay_state_floats(D, M));
#pragma unroll
                for (int x = 0; x < D; ++x)
#pragma unroll
                    for (int l = 0; l < CPL; ++l)
                        Mc[l][x] = A.rs[rs_at(base, lane_row<D, LPC>(x, sub) * M + col0 + l)];
#pragma unroll
                for (int r = 0; r < RPL; ++r)
#pragma unroll
                    for (int x = 0; x < D; ++x)
                        P[r][x] = A.rs[rs_at(base, D * M + tri_index(D, row0 + r, lane_row<D, LPC>(x, sub)))];
            } else {
                // written by this kernel in phase A: coherent loads
                float flat[G::kWsLane];
                load_vec_coherent<G::kWsLane>(ws + (j - 1) * kWsChain, flat);
#pragma unroll
                for (int l = 0; l < CPL; ++l)
#pragma unroll
                    for (int i = 0; i < D; ++i) Mc[l][i] = flat[l * D + i];
#pragma unroll
                for (int r = 0; r < RPL; ++r)
#pragma unroll
                    for (int jj = 0; jj < D; ++jj) P[r][jj] = flat[G::hMB + r * D + jj];
            }
            // the boundary checkpoint the next sub-chunk starts from: start its fetch now
            if (active && have_rs) {
                if (j == 1) {
                    prefetch_state_l2<LPC>(bm + ci * D * M, D * M, sub);
                    prefetch_state_l2<LPC>(bc + ci * D * D, D * D, sub);
                } else if (j == 0 && ci > 0 && (L + kS - 1) / kS <= 1) {
                    prefetch_state_l2<LPC>(bm + (ci - 1) * D * M, D * M, sub);
                    prefetch_state_l2<LPC>(bc + (ci - 1) * D * D, D * D, sub);
                }
            }
            // replay into history
            for (int tau = 0; tau < slen; ++tau) {
                {
                    float flat[G::hMB];
#pragma unroll
                    for (int l = 0; l < CPL; ++l)
#pragma unroll
                        for (int i = 0; i < D; ++i) flat[l * D + i] = Mc[l][i];
                    put_block<G::hMB, LPC>(hist + G::hM + tau * M * D, sub, flat);
                    float pf[G::hPB];
#pragma unroll
                    for (int r = 0; r < RPL; ++r)
#pragma unroll
                        for (int jj = 0; jj < D; ++jj) pf[r * D + jj] = P[r][jj];
                    put_block<G::hPB, LPC>(hist + G::hP + tau * D * D, sub, pf);
                }
                Tok<D, M, LPC> tk;
                read_tok<D, M, LPC, FIXED, TIn>(stage, c, tau, sub, tk);
                float u[D], u_own[RPL], e[CPL], beta, s;
                forward_step<D, M, LPC>(g, tk, floor_, Mc, P, u, u_own, e, beta, s);
                sts_vec<RPL>(hU_at(tau) + row0, u_own);
                sts_vec<CPL>(hE_at(tau) + col0, e);
                if (sub == 0) *reinterpret_cast<float2 *>(hB_at(tau)) = make_float2(beta, s);
            }
            __syncwarp();
            // Mc holds the post-update mean of the sub-chunk's last token; after
            // each reverse step Mn takes that step's pre-update mean
            float Mn[CPL][D];
#pragma unroll
            for (int l = 0; l < CPL; ++l)
#pragma unroll
                for (int i = 0; i < D; ++i) Mn[l][i] = Mc[l][i];
            for (int tau = slen - 1; tau >= 0; --tau) {
                const long row = chain * T + ci * L + static_cast<long>(j) * kS + tau;
                // row-indexed vectors in lane order: own rows at positions 0 .. RPL-1
                float k[D], a[D], q[D], u[D];
                lds_rows<D, LPC>(reinterpret_cast<const TIn *>(stage + G::oK + c * G::csK + tau * G::rbK), sub, k);
                lds_rows<D, LPC>(reinterpret_cast<const TIn *>(stage + G::oQ + c * G::csK + tau * G::rbK), sub, q);
                float p;
                if constexpr (FIXED) {
#pragma unroll
                    for (int jj = 0; jj < D; ++jj) a[jj] = kFixedDecay;
                    p = kFixedProcess;
                } else {
                    lds_rows<D, LPC>(reinterpret_cast<const float *>(stage + G::oA + c * G::csA + tau * G::rbA), sub, a);
                    p = reinterpret_cast<const float *>(stage + G::oP + c * G::csP)[tau];
                }
                lds_rows<D, LPC>(hU_at(tau), sub, u);
                const float2 bs = *reinterpret_cast<const float2 *>(hB_at(tau));
                const float beta = bs.x, s = bs.y;
                float e[CPL], gyv[CPL];
                lds_vec<CPL>(hE_at(tau) + col0, e);
                if (has_gy) {
                    lds_vec<CPL>(reinterpret_cast<const float *>(stage + G::oG + c * G::csG + tau * G::rbG) + col0,
                                 gyv);
                } else {
#pragma unroll
                    for (int l = 0; l < CPL; ++l) gyv[l] = 0.f;
                }
                float Mp[CPL][D], Pp[RPL][D];
                {
                    float flat[G::hMB];
                    get_block<G::hMB, LPC>(hist + G::hM + tau * M * D, sub, flat);
#pragma unroll
                    for (int l = 0; l < CPL; ++l)
#pragma unroll
                        for (int i = 0; i < D; ++i) Mp[l][i] = flat[l * D + i];
                    float pf[G::hPB];
                    get_block<G::hPB, LPC>(hist + G::hP + tau * D * D, sub, pf);
#pragma unroll
                    for (int r = 0; r < RPL; ++r)
#pragma unroll
                        for (int jj = 0; jj < D; ++jj) Pp[r][jj] = pf[r * D + jj];
                }

                // dL/d(post-update mean)
#pragma unroll
                for (int l = 0; l < CPL; ++l)
#pragma unroll
                    for (int i = 0; i < D; ++i) gM[l][i] = fmaf(q[i], gyv[l], gM[l][i]);
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
                float tot[4][RPL];
                if constexpr (NEED_DYN) {
                    g.template reduce_scatter_lane<4, RPL>(part, tot);
                } else {
                    float part3[3][D];
#pragma unroll
                    for (int v = 0; v < 3; ++v)
#pragma unroll
                        for (int i = 0; i < D; ++i) part3[v][i] = part[v][i];
                    float tot3[3][RPL];
                    g.template reduce_scatter_lane<3, RPL>(part3, tot3);
#pragma unroll
                    for (int r = 0; r < RPL; ++r) {
                        tot[0][r] = tot3[0][r];
                        tot[1][r] = tot3[1][r];
                        tot[2][r] = tot3[2][r];
                        tot[3][r] = 0.f;
                    }
                }

                float Ru[RPL];
                float trR = 0.f;
#pragma unroll
                for (int r = 0; r < RPL; ++r) {
                    float acc = 0.f;
#pragma unroll
                    for (int jj = 0; jj < D; ++jj) acc = fmaf(R[r][jj], u[jj], acc);
                    Ru[r] = acc;
                    gb = fmaf(-u[r], acc, gb);
                    if constexpr (NEED_DYN) trR += R[r][r];
                }
                if constexpr (NEED_DYN) {
#pragma unroll
                    for (int h = 1; h < LPC; h <<= 1) {
                        gb += g.xor_(gb, h);
                        trR += g.xor_(trR, h);
                    }
                } else {
                    gb = g.allsum(gb);
                }
                const float gs = (s >= floor_) ? -beta * beta * gb : 0.f;
                float gu_own[RPL];
#pragma unroll
                for (int r = 0; r < RPL; ++r) gu_own[r] = beta * tot[1][r] - 2.f * beta * Ru[r] + gs * k[r];
                float gu[D];
                g.template gather_lane<RPL>(gu_own, gu);

                float ag[D];
#pragma unroll
                for (int jj = 0; jj < D; ++jj) ag[jj] = a[jj] * gu[jj];
                float gk_own[RPL], ga_own[RPL];
#pragma unroll
                for (int r = 0; r < RPL; ++r) {
                    float z = 0.f;
#pragma unroll
                    for (int jj = 0; jj < D; ++jj) z = fmaf(Pp[r][jj], ag[jj], z);
                    const float gk3 = fmaf(a[r], z, p * gu_own[r]);
                    gk_own[r] = fmaf(-a[r], tot[2][r], fmaf(gs, u[r], gk3));
                    float gaP = 0.f;
#pragma unroll
                    for (int jj = 0; jj < D; ++jj) {
                        // rounded products and sum, never contracted: lanes
                        // owning rows i and j form bit-identical S_ij, S_ji
                        const float x = __fadd_rn(__fmul_rn(gu_own[r], k[jj]), __fmul_rn(gu[jj], k[r]));
                        const float Sj = fmaf(0.5f, x, R[r][jj]);
                        if constexpr (NEED_DYN) gaP = fmaf(Sj, a[jj] * Pp[r][jj], gaP);
                        R[r][jj] = (a[r] * a[jj]) * Sj;
                    }
                    ga_own[r] = fmaf(2.f, gaP, tot[3][r]);
                }
                float gpk = 0.f;
                if constexpr (NEED_DYN) {
#pragma unroll
                    for (int jj = 0; jj < D; ++jj) gpk = fmaf(gu[jj], k[jj], gpk);
                }
                if (active) {
                    float gq_own[RPL];
#pragma unroll
                    for (int r = 0; r < RPL; ++r) gq_own[r] = tot[0][r];
                    store_vec<RPL>(A.gk + row * D + row0, gk_own);
                    store_vec<RPL>(A.gq + row * D + row0, gq_own);
                    store_vec<CPL>(A.gv + row * M + col0, ge);
                    if constexpr (NEED_DYN) {
                        if constexpr (FIXED) {
                            float z[RPL];
#pragma unroll
                            for (int r = 0; r < RPL; ++r) z[r] = 0.f;
                            store_vec<RPL>(A.ga + row * D + row0, z);
                            if (sub == 0) {
                                A.gp[row] = 0.f;
                                A.gr[row] = 0.f;
                            }
                        } else {
                            store_vec<RPL>(A.ga + row * D + row0, ga_own);
                            if (sub == 0) {
                                A.gp[row] = trR + gpk;
                                A.gr[row] = gs;
                            }
                        }
                    }
                }
#pragma unroll
                for (int l = 0; l < CPL; ++l)
#pragma unroll
                    for (int i = 0; i < D; ++i) Mn[l][i] = Mp[l][i];
            }
            __syncwarp();
            ++qc;
        }
    }
    cp_async_wait<0>();
    if constexpr (NEED_INIT) {
        if (active) {
            stg_mean_cols<D, M, LPC>(A.gm0 + chain * D * M, col0, sub, gM);
#pragma unroll
            for (int r = 0; r < RPL; ++r) stg_row<D, LPC>(A.gc0 + chain * D * D + (row0 + r) * D, sub, R[r]);
        }
    }
}

// ===========================================================================
// Host launchers
// ===========================================================================
template <int D, int M, int LPC, typename TIn>
constexpr size_t fwd_smem() {
    return static_cast<size_t>(kStagesFwd) * Geo<D, M, LPC, TIn>::kTile;
}
template <int D, int M, int LPC, typename TIn>
constexpr size_t bwd_smem() {
    using G = Geo<D, M, LPC, TIn>;
    return static_cast<size_t>(kStagesBwd) * G::kTile + static_cast<size_t>(G::kHistAll) * sizeof(float);
}

template <int D, int M, int LPC, bool FIXED, typename TIn>
int launch_forward(const FwdArgs<TIn> &a, cudaStream_t st) {
    if (a.n == 0) return BSSM_OK;
    constexpr int C = Geo<D, M, LPC, TIn>::C;
    const long blocks = (a.n + C - 1) / C;
    if (blocks > 0x7fffffffL) return fail(BSSM_ERR_INVALID, "too many chains");
    constexpr size_t smem = fwd_smem<D, M, LPC, TIn>();
    auto kern = forward_staged<D, M, LPC, FIXED, TIn>;
    if (smem > 48 * 1024) {
        cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (err != cudaSuccess) return fail(BSSM_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
    }
    kern<<<static_cast<unsigned>(blocks), 32, smem, st>>>(a);
    return check_launch("forward_staged");
}

template <int D, int M, int LPC, bool FIXED, bool NEED_DYN, bool NEED_INIT, typename TIn>
int launch_backward_impl(const BwdArgs<TIn> &a, cudaStream_t st) {
    constexpr int C = Geo<D, M, LPC, TIn>::C;
    const long blocks = (a.n + C - 1) / C;
    if (blocks > 0x7fffffffL) return fail(BSSM_ERR_INVALID, "too many chains");
    constexpr size_t smem = bwd_smem<D, M, LPC, TIn>();
    auto kern = backward_staged<D, M, LPC, FIXED, NEED_DYN, NEED_INIT, TIn>;
    if (smem > 48 * 1024) {
        cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (err != cudaSuccess) return fail(BSSM_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
    }
    kern<<<static_cast<unsigned>(blocks), 32, smem, st>>>(a);
    return check_launch("backward_staged");
}

template <int D, int M, int LPC, bool FIXED, typename TIn>
int launch_backward(const BwdArgs<TIn> &a, bool dyn, bool init, cudaStream_t st) {
    if (dyn && init) return launch_backward_impl<D, M, LPC, FIXED, true, true, TIn>(a, st);
    if (dyn) return launch_backward_impl<D, M, LPC, FIXED, true, false, TIn>(a, st);
    if (init) return launch_backward_impl<D, M, LPC, FIXED, false, true, TIn>(a, st);
    return launch_backward_impl<D, M, LPC, FIXED, false, false, TIn>(a, st);
}

// Lanes per chain used for each key dimension.
template <int D>
struct Lanes {
    static constexpr int kFwd = D >= 8 ? 4 : D;
    static constexpr int kBwd = D >= 8 ? 4 : D;
};

template <int D, typename TIn>
int forward_d(int fixed, const FwdArgs<TIn> &a, cudaStream_t st) {
    constexpr int LPC = Lanes<D>::kFwd;
    return fixed ? launch_forward<D, 8, LPC, true, TIn>(a, st) : launch_forward<D, 8, LPC, false, TIn>(a, st);
}
template <int D, typename TIn>
int backward_d(int fixed, bool dyn, bool init, const BwdArgs<TIn> &a, cudaStream_t st) {
    constexpr int LPC = Lanes<D>::kBwd;
    return fixed ? launch_backward<D, 8, LPC, true, TIn>(a, dyn, init, st)
                 : launch_backward<D, 8, LPC, false, TIn>(a, dyn, init, st);
}

}  // namespace staged

template <typename TIn>
bool staged_supported(int d) {
    // cp.async moves rows of >= 4 bytes: every (D, dtype) except D = 1 with
    // 16-bit keys/queries qualifies.
    return d == 8 || d == 4 || d == 2 || (d == 1 && sizeof(TIn) == 4);
}

template <typename TIn>
int staged_forward(int d, int fixed, const FwdArgs<TIn> &a, cudaStream_t st) {
    switch (d) {
        case 1: if constexpr (sizeof(TIn) == 4) return staged::forward_d<1, TIn>(fixed, a, st); break;
        case 2: return staged::forward_d<2, TIn>(fixed, a, st);
        case 4: return staged::forward_d<4, TIn>(fixed, a, st);
        case 8: return staged::forward_d<8, TIn>(fixed, a, st);
    }
    return fail(BSSM_ERR_UNSUPPORTED, "staged forward: key_dim %d", d);
}

template <typename TIn>
int staged_backward(int d, int fixed, bool dyn, bool init, const BwdArgs<TIn> &a, cudaStream_t st) {
    switch (d) {
        case 1: if constexpr (sizeof(TIn) == 4) return staged::backward_d<1, TIn>(fixed, dyn, init, a, st); break;
        case 2: return staged::backward_d<2, TIn>(fixed, dyn, init, a, st);
        case 4: return staged::backward_d<4, TIn>(fixed, dyn, init, a, st);
        case 8: return staged::backward_d<8, TIn>(fixed, dyn, init, a, st);
    }
    return fail(BSSM_ERR_UNSUPPORTED, "staged backward: key_dim %d", d);
}

template bool staged_supported<float>(int);
template bool staged_supported<__nv_bfloat16>(int);
template int staged_forward<float>(int, int, const FwdArgs<float> &, cudaStream_t);
template int staged_forward<__nv_bfloat16>(int, int, const FwdArgs<__nv_bfloat16> &, cudaStream_t);
template int staged_backward<float>(int, int, bool, bool, const BwdArgs<float> &, cudaStream_t);
template int staged_backward<__nv_bfloat16>(int, int, bool, bool, const BwdArgs<__nv_bfloat16> &, cudaStream_t);

}  // namespace bssm
