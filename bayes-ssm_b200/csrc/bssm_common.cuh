// bssm_common.cuh -- device helpers shared by the Bayesian-layer kernels.
//
// A "chain" is one independent (batch, head) sequence.  A chain is served by
// a group of LPC consecutive lanes of one warp; the group's lane mask keeps
// every shuffle and __syncwarp inside the group, so whole groups may retire
// early (a partial last CTA) without stalling the rest of the warp.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace bssm {

template <int LPC>
struct LaneGroup {
    static_assert(LPC == 1 || LPC == 2 || LPC == 4 || LPC == 8 || LPC == 16 || LPC == 32,
                  "lanes per chain must divide the warp");
    unsigned mask;
    int sub;  // rank inside the group

    __device__ __forceinline__ LaneGroup() {
        const int lane = threadIdx.x & 31;
        sub = lane & (LPC - 1);
        mask = (LPC == 32) ? 0xffffffffu : (((1u << LPC) - 1u) << (lane - sub));
    }
    // value of `v` held by group rank `src`
    __device__ __forceinline__ float bcast(float v, int src) const {
        if constexpr (LPC == 1) {
            return v;
        } else {
            return __shfl_sync(mask, v, src, LPC);
        }
    }
    __device__ __forceinline__ float xor_(float v, int h) const {
        return __shfl_xor_sync(mask, v, h, LPC);
    }
    // sum over the group, result in every lane
    __device__ __forceinline__ float allsum(float v) const {
#pragma unroll
        for (int h = 1; h < LPC; h <<= 1) v += xor_(v, h);
        return v;
    }
    __device__ __forceinline__ void sync() const {
        if constexpr (LPC > 1) __syncwarp(mask);
    }
    // Gather: out[j] = v of rank j, j < LPC.
    template <int N>
    __device__ __forceinline__ void gather(float v, float (&out)[N]) const {
        static_assert(N == LPC, "gather size");
#pragma unroll
        for (int j = 0; j < N; ++j) out[j] = bcast(v, j);
    }
    // Reduce-scatter of NV vectors of LPC partial sums: after the call, lane
    // `sub` holds in out[v] the group total of element `sub` of vector v.
    // Recursive halving: log2(LPC) stages, LPC-1 shuffles per vector.
    template <int NV>
    __device__ __forceinline__ void reduce_scatter(float (&vals)[NV][LPC], float (&out)[NV]) const {
        if constexpr (LPC == 1) {
#pragma unroll
            for (int v = 0; v < NV; ++v) out[v] = vals[v][0];
        } else {
#pragma unroll
            for (int h = LPC / 2; h >= 1; h >>= 1) {
                const bool upper = (sub & h) != 0;
#pragma unroll
                for (int x = 0; x < h; ++x) {
#pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        const float lo = vals[v][x], hi = vals[v][x + h];
                        const float send = upper ? lo : hi;
                        const float keep = upper ? hi : lo;
                        vals[v][x] = keep + xor_(send, h);
                    }
                }
            }
#pragma unroll
            for (int v = 0; v < NV; ++v) out[v] = vals[v][0];
        }
    }
    // Row gather: lane `sub` owns RPL consecutive entries (rows sub*RPL ..);
    // out receives all LPC*RPL entries in row order.
    template <int RPL>
    __device__ __forceinline__ void gather_rows(const float (&own)[RPL], float (&out)[LPC * RPL]) const {
#pragma unroll
        for (int src = 0; src < LPC; ++src)
#pragma unroll
            for (int r = 0; r < RPL; ++r) out[src * RPL + r] = bcast(own[r], src);
    }
    // Gather into lane-relative row order (see bssm_staged.cu): position x
    // receives row x ^ (sub*RPL), owned by rank (x/RPL) ^ sub at its slot x%RPL.
    template <int RPL>
    __device__ __forceinline__ void gather_lane(const float (&own)[RPL], float (&out)[LPC * RPL]) const {
#pragma unroll
        for (int x = 0; x < LPC * RPL; ++x) out[x] = bcast(own[x % RPL], (x / RPL) ^ sub);
    }
    // Reduce-scatter of NV vectors held in lane-relative row order: at the
    // stage with partner distance h a lane keeps positions [0, h*RPL) and its
    // partner's positions [h*RPL, 2h*RPL) hold the same rows, so no selects
    // are needed.  Lane `sub` ends with the totals of its own rows in
    // positions 0 .. RPL-1.
    template <int NV, int RPL>
    __device__ __forceinline__ void reduce_scatter_lane(float (&vals)[NV][LPC * RPL],
                                                        float (&out)[NV][RPL]) const {
#pragma unroll
        for (int h = LPC / 2; h >= 1; h >>= 1)
#pragma unroll
            for (int x = 0; x < h * RPL; ++x)
#pragma unroll
                for (int v = 0; v < NV; ++v) vals[v][x] += xor_(vals[v][x + h * RPL], h);
#pragma unroll
        for (int v = 0; v < NV; ++v)
#pragma unroll
            for (int r = 0; r < RPL; ++r) out[v][r] = vals[v][r];
    }
    // Reduce-scatter of NV vectors of LPC*RPL partial sums: lane `sub` ends
    // with the group totals of entries sub*RPL .. sub*RPL+RPL-1 of each vector.
    // Recursive halving: at the stage with partner distance h the lanes with
    // bit h set keep the upper half of their current window.
    template <int NV, int RPL>
    __device__ __forceinline__ void reduce_scatter_rows(float (&vals)[NV][LPC * RPL],
                                                        float (&out)[NV][RPL]) const {
        if constexpr (LPC > 1) {
#pragma unroll
            for (int h = LPC / 2; h >= 1; h >>= 1) {
                const bool upper = (sub & h) != 0;
#pragma unroll
                for (int x = 0; x < h * RPL; ++x) {
#pragma unroll
                    for (int v = 0; v < NV; ++v) {
                        const float lo = vals[v][x], hi = vals[v][x + h * RPL];
                        const float send = upper ? lo : hi;
                        const float keep = upper ? hi : lo;
                        vals[v][x] = keep + xor_(send, h);
                    }
                }
            }
        }
#pragma unroll
        for (int v = 0; v < NV; ++v)
#pragma unroll
            for (int r = 0; r < RPL; ++r) out[v][r] = vals[v][r];
    }
};

// v[idx] for a runtime idx without dynamic register indexing.
template <int N>
__device__ __forceinline__ float pick(const float (&v)[N], int idx) {
    float r = v[0];
#pragma unroll
    for (int j = 1; j < N; ++j) r = (idx == j) ? v[j] : r;
    return r;
}

// ---------------------------------------------------------------------------
// Vector loads / stores of N consecutive elements (N in {1,2,4,8}).  bf16 is
// the upper half of an IEEE float32, so widening is a 16-bit shift.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

template <int N>
__device__ __forceinline__ void load_vec(const float *__restrict__ p, float (&o)[N]) {
    if constexpr (N % 4 == 0) {
#pragma unroll
        for (int i = 0; i < N; i += 4) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(p + i));
            o[i] = v.x; o[i + 1] = v.y; o[i + 2] = v.z; o[i + 3] = v.w;
        }
    } else if constexpr (N == 2) {
        const float2 v = __ldg(reinterpret_cast<const float2 *>(p));
        o[0] = v.x; o[1] = v.y;
    } else {
        static_assert(N == 1, "vector width");
        o[0] = __ldg(p);
    }
}

template <int N>
__device__ __forceinline__ void load_vec(const __nv_bfloat16 *__restrict__ p, float (&o)[N]) {
    if constexpr (N == 8) {
        const uint4 w = __ldg(reinterpret_cast<const uint4 *>(p));
        o[0] = bf16_lo(w.x); o[1] = bf16_hi(w.x); o[2] = bf16_lo(w.y); o[3] = bf16_hi(w.y);
        o[4] = bf16_lo(w.z); o[5] = bf16_hi(w.z); o[6] = bf16_lo(w.w); o[7] = bf16_hi(w.w);
    } else if constexpr (N == 4) {
        const uint2 w = __ldg(reinterpret_cast<const uint2 *>(p));
        o[0] = bf16_lo(w.x); o[1] = bf16_hi(w.x); o[2] = bf16_lo(w.y); o[3] = bf16_hi(w.y);
    } else if constexpr (N == 2) {
        const uint32_t w = __ldg(reinterpret_cast<const unsigned int *>(p));
        o[0] = bf16_lo(w); o[1] = bf16_hi(w);
    } else {
        static_assert(N == 1, "vector width");
        const unsigned short h = __ldg(reinterpret_cast<const unsigned short *>(p));
        o[0] = __uint_as_float(static_cast<uint32_t>(h) << 16);
    }
}

template <int N>
__device__ __forceinline__ void store_vec(float *__restrict__ p, const float (&v)[N]) {
    if constexpr (N % 4 == 0) {
#pragma unroll
        for (int i = 0; i < N; i += 4)
            *reinterpret_cast<float4 *>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else if constexpr (N == 2) {
        *reinterpret_cast<float2 *>(p) = make_float2(v[0], v[1]);
    } else {
        static_assert(N == 1, "vector width");
        p[0] = v[0];
    }
}

template <int N>
__device__ __forceinline__ void store_vec(__nv_bfloat16 *__restrict__ p, const float (&v)[N]) {
    if constexpr (N % 2 == 0) {
#pragma unroll
        for (int i = 0; i < N; i += 2)
            *reinterpret_cast<__nv_bfloat162 *>(p + i) = __floats2bfloat162_rn(v[i], v[i + 1]);
    } else {
        static_assert(N == 1, "vector width");
        p[0] = __float2bfloat16_rn(v[0]);
    }
}

__device__ __forceinline__ void store_one(float *p, float v) { *p = v; }
__device__ __forceinline__ void store_one(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

}  // namespace bssm

namespace bssm {

// ---------------------------------------------------------------------------
// Asynchronous global -> shared copies (cp.async, L2-only for 16-byte pieces).
// ---------------------------------------------------------------------------
template <int G>
__device__ __forceinline__ void cp_async(uint32_t smem_addr, const void *gptr) {
    static_assert(G == 4 || G == 8 || G == 16, "cp.async piece size");
    if constexpr (G == 16) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr), "l"(gptr) : "memory");
    } else {
        asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(smem_addr), "l"(gptr), "n"(G)
                     : "memory");
    }
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// N consecutive elements from shared memory, widened to float.
template <int N>
__device__ __forceinline__ void lds_vec(const float *p, float (&o)[N]) {
    if constexpr (N % 4 == 0) {
#pragma unroll
        for (int i = 0; i < N; i += 4) {
            const float4 v = *reinterpret_cast<const float4 *>(p + i);
            o[i] = v.x; o[i + 1] = v.y; o[i + 2] = v.z; o[i + 3] = v.w;
        }
    } else if constexpr (N == 2) {
        const float2 v = *reinterpret_cast<const float2 *>(p);
        o[0] = v.x; o[1] = v.y;
    } else {
        static_assert(N == 1, "width");
        o[0] = p[0];
    }
}
template <int N>
__device__ __forceinline__ void lds_vec(const __nv_bfloat16 *p, float (&o)[N]) {
    if constexpr (N % 8 == 0) {
#pragma unroll
        for (int i = 0; i < N; i += 8) {
            const uint4 w = *reinterpret_cast<const uint4 *>(p + i);
            o[i] = bf16_lo(w.x); o[i + 1] = bf16_hi(w.x); o[i + 2] = bf16_lo(w.y); o[i + 3] = bf16_hi(w.y);
            o[i + 4] = bf16_lo(w.z); o[i + 5] = bf16_hi(w.z); o[i + 6] = bf16_lo(w.w); o[i + 7] = bf16_hi(w.w);
        }
    } else if constexpr (N == 4) {
        const uint2 w = *reinterpret_cast<const uint2 *>(p);
        o[0] = bf16_lo(w.x); o[1] = bf16_hi(w.x); o[2] = bf16_lo(w.y); o[3] = bf16_hi(w.y);
    } else if constexpr (N == 2) {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(p);
        o[0] = bf16_lo(w); o[1] = bf16_hi(w);
    } else {
        static_assert(N == 1, "width");
        const unsigned short h = *reinterpret_cast<const unsigned short *>(p);
        o[0] = __uint_as_float(static_cast<uint32_t>(h) << 16);
    }
}

template <int N>
__device__ __forceinline__ void sts_vec(float *p, const float (&v)[N]) {
    if constexpr (N % 4 == 0) {
#pragma unroll
        for (int i = 0; i < N; i += 4)
            *reinterpret_cast<float4 *>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else if constexpr (N == 2) {
        *reinterpret_cast<float2 *>(p) = make_float2(v[0], v[1]);
    } else {
        static_assert(N == 1, "width");
        p[0] = v[0];
    }
}

}  // namespace bssm
