// bssm_assoc_scan.cu -- static associative scan (A = I, Q = 0) for sm_100a.
//
// Information form (catid/bayes-ssm bayes_ssm/replay_ssm.py:155-270):
//   Lambda_t = inv(P0) + sum_{s<=t} k_s k_s^T / r_s,
//   N_t      = inv(P0) M0 + sum_{s<=t} k_s v_s^T / r_s,
//   M_t = Lambda_t^{-1} N_t,  y_t = M_t^T q_t,  P_T = Lambda_T^{-1}.
// The reference symmetrises Lambda_t and uses a Cholesky factor; so does
// this kernel.  Because only y_t is needed at every t, each token solves
// Lambda_t x = q_t for one right-hand side and reads y_t = N_t^T x, instead of
// solving for the full D x M mean; M_T and P_T are formed once, at T-1.
//
// Grid: (ceil(T / 8), N).  A CTA of 8 warps owns 8 consecutive tokens of one
// chain.  The CTA first forms the prefix base at its first token (all
// earlier tokens, summed cooperatively entry by entry), stages its 8 tokens in
// shared memory, then warp w factors Lambda_{t0+w} (left-looking Cholesky,
// lane = row) and runs the two triangular solves with shuffles.
// Limits: key_dim <= 32 (one lane per row), value_dim <= 256.
#include <cstdarg>
#include <cstdio>
#include <string>

#include "bayes_ssm_b200.h"
#include "bssm_common.cuh"
#include "bssm_internal.h"

namespace bssm {

constexpr int kScanWarps = 8;
constexpr int kScanThreads = kScanWarps * 32;
constexpr int kScanMaxD = 32;
constexpr int kScanMaxM = 256;
constexpr int kScanChunk = 32;  // prefix tokens staged per round

// status bits written by the kernel
constexpr int kScanNotPD = 1;       // a Cholesky pivot was <= 0 or not finite
constexpr int kScanBadVariance = 2; // an observation variance was < floor or not finite

struct ScanArgs {
    const float *keys, *values, *queries, *obs, *mean0, *cov0;
    float *out, *mean_final, *cov_final;
    int *status;
    long n, t;
    int d, m;
    float floor;
};

// Left-looking Cholesky of the D x D matrix in A, rows `ld` floats apart (ld
// = D + 1 keeps a warp's row-per-lane accesses on distinct banks); the lower
// triangle receives L.  Lane i owns row i.  Returns false (in every lane)
// when a pivot is not positive.
__device__ bool warp_cholesky(float *A, int D, int ld, int lane) {
    bool ok = true;
    for (int j = 0; j < D; ++j) {
        if (lane == j) {
            float s = A[j * ld + j];
            for (int k = 0; k < j; ++k) s = fmaf(-A[j * ld + k], A[j * ld + k], s);
            const bool good = s > 0.f && s < 3.0e38f;
            A[j * ld + j] = good ? sqrtf(s) : -1.f;  // -1 marks a failed pivot
        }
        __syncwarp();
        const float piv = A[j * ld + j];
        ok = ok && (piv > 0.f);
        const float rpiv = 1.0f / piv;  // one division per column
        if (lane > j && lane < D) {
            float z = A[lane * ld + j];
            for (int k = 0; k < j; ++k) z = fmaf(-A[lane * ld + k], A[j * ld + k], z);
            A[lane * ld + j] = z * rpiv;
        }
        __syncwarp();
    }
    return ok;
}

// Solve (L L^T) x = b for one right-hand side; lane i holds b_i / x_i.
// Each lane takes the reciprocal of its own pivot once, so the serial
// substitution steps multiply instead of divide.
__device__ float warp_chol_solve(const float *L, int D, int ld, int lane, float b) {
    const float rdi = lane < D ? 1.0f / L[lane * ld + lane] : 0.f;
    float z = 0.f;
    for (int k = 0; k < D; ++k) {  // forward: L z = b
        const float zk = __shfl_sync(0xffffffffu, b * rdi, k);
        if (lane == k) z = zk;
        if (lane > k && lane < D) b = fmaf(-L[lane * ld + k], zk, b);
    }
    float x = 0.f;
    for (int k = D - 1; k >= 0; --k) {  // backward: L^T x = z
        const float xk = __shfl_sync(0xffffffffu, z * rdi, k);
        if (lane == k) x = xk;
        if (lane < k) z = fmaf(-L[k * ld + lane], xk, z);
    }
    return x;
}

// (L L^T)^{-1} from the Cholesky factor L (rows `ld` apart), by the whole
// CTA, in rolled loops (this runs once per CTA, so straight-line code would
// cost more in instruction fetch than it saves).  Thread c < D forms column c
// of L^{-1} by forward substitution into `linv`; then each entry
// out_ij = sum_{k >= max(i,j)} Linv_ki Linv_kj, which is exactly symmetric
// because the products commute.  `rd` receives 1 / L_ii.  Contains
// __syncthreads: every thread of the CTA calls it.
__device__ void block_chol_inverse(const float *L, int D, int ld, float *linv, float *rd, float *out,
                                   int ldo, int tid) {
    if (tid < D) rd[tid] = 1.0f / L[tid * ld + tid];
    __syncthreads();
    if (tid < D) {
        const int c = tid;
        for (int i = 0; i < c; ++i) linv[i * ld + c] = 0.f;
        linv[c * ld + c] = rd[c];
        for (int i = c + 1; i < D; ++i) {
            float s = 0.f;
            for (int k = c; k < i; ++k) s = fmaf(-L[i * ld + k], linv[k * ld + c], s);
            linv[i * ld + c] = s * rd[i];
        }
    }
    __syncthreads();
    for (int e = tid; e < D * D; e += kScanThreads) {
        const int i = e / D, j = e % D;
        float acc = 0.f;
        for (int k = i > j ? i : j; k < D; ++k) acc = fmaf(linv[k * ld + i], linv[k * ld + j], acc);
        out[i * ldo + j] = acc;
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kScanThreads) assoc_scan_kernel(const ScanArgs A) {
    extern __shared__ __align__(16) float sm[];
    const int D = A.d, M = A.m;
    const long chain = blockIdx.y;
    const long t0 = static_cast<long>(blockIdx.x) * kScanWarps;
    const long T = A.t;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nblock = static_cast<int>((T - t0) < kScanWarps ? (T - t0) : kScanWarps);

    const int LD = D + 1;            // row stride of the D x D matrices
    float *lam = sm;                 // D*LD  prefix precision before t0
    float *nat = lam + D * LD;       // D*M   prefix natural parameter before t0
    float *bk = nat + D * M;         // 8*D   block keys
    float *bw = bk + kScanWarps * D; // 8*D   block keys / r
    float *bv = bw + kScanWarps * D; // 8*M   block values
    float *ptm = bv + kScanWarps * M;                 // D*LD  P_T (last block only)
    float *wsc = ptm + D * LD;                        // per warp: D*LD + 2*D + 8
    float *mine = wsc + warp * (D * LD + 2 * D + kScanWarps);
    float *xv = mine + D * LD;       // D   solution x
    float *dots = xv + D;            // 8   w_s . x
    float *stg = wsc + kScanWarps * (D * LD + 2 * D + kScanWarps);  // prefix chunk: keys, keys / r, values
    float *sk = stg, *sw = sk + kScanChunk * D, *sv = sw + kScanChunk * D;
    const float *kc = A.keys + chain * T * D;
    const float *vc = A.values + chain * T * M;
    const float *rc = A.obs + chain * T;

    // ---- 1. Lambda_0 = inv(sym(P0)), N_0 = Lambda_0 M0 (identity / zero defaults)
    if (A.cov0 == nullptr) {
        for (int e = tid; e < D * D; e += kScanThreads) lam[(e / D) * LD + e % D] = (e / D == e % D) ? 1.f : 0.f;
        for (int e = tid; e < D * M; e += kScanThreads)
            nat[e] = A.mean0 ? A.mean0[chain * D * M + e] : 0.f;
        __syncthreads();
    } else {
        const float *c0 = A.cov0 + chain * D * D;
        if (warp == 0) {
            for (int e = lane; e < D * D; e += 32) mine[(e / D) * LD + e % D] = 0.5f * (c0[e] + c0[(e % D) * D + e / D]);
            __syncwarp();
            if (!warp_cholesky(mine, D, LD, lane)) {
                if (lane == 0) atomicOr(A.status, kScanNotPD);
            }
        }
        __syncthreads();
        // Lambda_0 (exactly symmetric); L^{-1} and 1/L_ii in the prefix staging area
        block_chol_inverse(wsc, D, LD, stg, stg + D * LD, lam, LD, tid);  // wsc: warp 0's factor
        for (int e = tid; e < D * M; e += kScanThreads) {
            const int i = e / M, c = e % M;
            float acc = 0.f;
            if (A.mean0)
                for (int j = 0; j < D; ++j) acc = fmaf(lam[i * LD + j], A.mean0[chain * D * M + j * M + c], acc);
            nat[e] = acc;
        }
        __syncthreads();
    }

    // ---- 2. add every token before t0: chunks of kScanChunk tokens staged in
    // shared memory (one division per key element), then entry-parallel sums
    for (long s0 = 0; s0 < t0; s0 += kScanChunk) {
        const int ns = static_cast<int>((t0 - s0) < kScanChunk ? (t0 - s0) : kScanChunk);
        __syncthreads();  // the previous chunk is consumed
        for (int e = tid; e < ns * D; e += kScanThreads) {
            const float kv = kc[s0 * D + e];
            sk[e] = kv;
            sw[e] = kv / rc[s0 + e / D];
        }
        for (int e = tid; e < ns * M; e += kScanThreads) sv[e] = vc[s0 * M + e];
        __syncthreads();
        for (int e = tid; e < D * D + D * M; e += kScanThreads) {
            float acc = 0.f;
            if (e < D * D) {
                const int i = e / D, j = e % D;
                for (int s = 0; s < ns; ++s) acc = fmaf(sk[s * D + i], sw[s * D + j], acc);
                lam[i * LD + j] += acc;
            } else {
                const int i = (e - D * D) / M, c = (e - D * D) % M;
                for (int s = 0; s < ns; ++s) acc = fmaf(sw[s * D + i], sv[s * M + c], acc);
                nat[e - D * D] += acc;
            }
        }
    }
    // ---- 3. stage this block's tokens
    for (int e = tid; e < nblock * D; e += kScanThreads) {
        const int s = e / D, i = e % D;
        const float r = rc[t0 + s];
        if (!(r >= A.floor) || !isfinite(r)) atomicOr(A.status, kScanBadVariance);
        bk[e] = kc[(t0 + s) * D + i];
        bw[e] = kc[(t0 + s) * D + i] / r;
    }
    for (int e = tid; e < nblock * M; e += kScanThreads) bv[e] = vc[(t0 + e / M) * M + e % M];
    __syncthreads();

    // ---- 4. warp w: token t0 + w
    if (warp < nblock) {
        const long t = t0 + warp;
        for (int e = lane; e < D * D; e += 32) {
            const int i = e / D, j = e % D;
            float lij = lam[i * LD + j], lji = lam[j * LD + i];
            for (int s = 0; s <= warp; ++s) {
                lij = fmaf(bk[s * D + i], bw[s * D + j], lij);
                lji = fmaf(bk[s * D + j], bw[s * D + i], lji);
            }
            mine[i * LD + j] = 0.5f * (lij + lji);
        }
        __syncwarp();
        if (!warp_cholesky(mine, D, LD, lane)) {
            if (lane == 0) atomicOr(A.status, kScanNotPD);
        }
        const float qi = lane < D ? A.queries[(chain * T + t) * D + lane] : 0.f;
        const float x = warp_chol_solve(mine, D, LD, lane, qi);
        if (lane < D) xv[lane] = x;
        __syncwarp();
        if (lane <= warp) {
            float acc = 0.f;
            for (int i = 0; i < D; ++i) acc = fmaf(bw[lane * D + i], xv[i], acc);
            dots[lane] = acc;
        }
        __syncwarp();
        for (int c = lane; c < M; c += 32) {
            float y = 0.f;
            for (int i = 0; i < D; ++i) y = fmaf(nat[i * M + c], xv[i], y);
            for (int s = 0; s <= warp; ++s) y = fmaf(dots[s], bv[s * M + c], y);
            A.out[(chain * T + t) * M + c] = y;
        }
    }
    // ---- 5. final state, by the CTA that holds T-1: P_T = Lambda_T^{-1}
    // from the last warp's factor, N_T = N_{t0} + this block's tokens,
    // M_T = P_T N_T
    if (t0 + nblock == T) {
        __syncthreads();
        const float *lf = wsc + (nblock - 1) * (D * LD + 2 * D + kScanWarps);
        float *ntm = stg, *linv = ntm + D * M, *rd = linv + D * LD;
        for (int e = tid; e < D * M; e += kScanThreads) {
            const int i = e / M, c = e % M;
            float acc = nat[e];
            for (int s = 0; s < nblock; ++s) acc = fmaf(bw[s * D + i], bv[s * M + c], acc);
            ntm[e] = acc;
        }
        block_chol_inverse(lf, D, LD, linv, rd, ptm, LD, tid);
        for (int e = tid; e < D * D; e += kScanThreads)
            A.cov_final[chain * D * D + e] = ptm[(e / D) * LD + e % D];
        for (int e = tid; e < D * M; e += kScanThreads) {
            const int i = e / M, c = e % M;
            float acc = 0.f;
            for (int j = 0; j < D; ++j) acc = fmaf(ptm[i * LD + j], ntm[j * M + c], acc);
            A.mean_final[chain * D * M + e] = acc;
        }
    }
}


}  // namespace bssm

using namespace bssm;

extern "C" {

int bssm_assoc_scan_ex(int key_dim, int value_dim, const float *keys, const float *values,
                       const float *queries, const float *observation, const float *mean0,
                       const float *cov0, float *out, float *mean_final, float *cov_final,
                       int *status, long n, long t, double denominator_floor, void *stream) {
    if (key_dim <= 0 || key_dim > kScanMaxD || value_dim <= 0 || value_dim > kScanMaxM)
        return fail(BSSM_ERR_UNSUPPORTED, "assoc scan supports 1 <= key_dim <= %d and 1 <= value_dim <= %d "
                    "(got %d, %d)", kScanMaxD, kScanMaxM, key_dim, value_dim);
    if (n < 0 || t < 0) return fail(BSSM_ERR_INVALID, "negative size");
    if (!(denominator_floor > 0.0)) return fail(BSSM_ERR_INVALID, "denominator_floor must be positive");
    if (n == 0 || t == 0) {
        g_last_error.clear();
        return BSSM_OK;
    }
    if (!keys || !values || !queries || !observation || !out || !mean_final || !cov_final || !status)
        return fail(BSSM_ERR_INVALID, "assoc scan: null pointer");
    if (n > 65535) return fail(BSSM_ERR_INVALID, "assoc scan: at most 65535 chains per call");
    const long blocks_t = (t + kScanWarps - 1) / kScanWarps;
    if (blocks_t > 0x7fffffffL) return fail(BSSM_ERR_INVALID, "assoc scan: sequence too long");
    const int D = key_dim, M = value_dim;
    const int LD = D + 1;
    const size_t smem = sizeof(float) * static_cast<size_t>(
        D * LD + D * M + kScanWarps * (2 * D + M) + D * LD + kScanWarps * (D * LD + 2 * D + kScanWarps) +
        kScanChunk * (2 * D + M));
    if (smem > 48 * 1024) {
        cudaError_t err = cudaFuncSetAttribute(assoc_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
        if (err != cudaSuccess) return fail(BSSM_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(err));
    }
    ScanArgs a{keys, values, queries, observation, mean0, cov0, out, mean_final, cov_final, status,
               n, t, D, M, static_cast<float>(denominator_floor)};
    dim3 grid(static_cast<unsigned>(blocks_t), static_cast<unsigned>(n));
    assoc_scan_kernel<<<grid, kScanThreads, smem, static_cast<cudaStream_t>(stream)>>>(a);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return fail(BSSM_ERR_CUDA, "assoc_scan_kernel: %s", cudaGetErrorString(err));
    g_last_error.clear();
    return BSSM_OK;
}

}  // extern "C"
