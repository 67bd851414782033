// bssm_tmem.cuh -- tensor-memory (TMEM) helpers for sm_100a.
//
// TMEM is 128 lanes x 512 columns of 32-bit cells per SM.  Warp w of a CTA
// reaches lanes 32*(w%4) .. 32*(w%4)+31; with the 32x32b shape each thread of
// the warp reads or writes its own lane, N consecutive columns per
// instruction (.x1 .. .x32).  A TMEM address is (lane << 16) | column.
//
// The kernels use TMEM as per-thread scratch: thread = lane = chain.  The
// wrappers below are the PTX instructions tcgen05.{alloc,dealloc,
// relinquish_alloc_permit,ld,st,wait,fence} written out; the destination
// registers of tcgen05.ld are defined only after tcgen05.wait::ld, so every
// load helper here ends with the wait and ties its outputs to it.
#pragma once

#include <stdint.h>

namespace bssm {
namespace tmem {

// ---- allocation (one full warp; the address lands in shared memory) --------
__device__ __forceinline__ void alloc(uint32_t *smem_slot, uint32_t ncols) {
    const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem_slot));
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Order tcgen05 operations against a thread barrier (before / after it).
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- raw 32x32b loads / stores ----------------------------------------------
__device__ __forceinline__ void tmem_ld_x1(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];"
                 : "=r"(r[0])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_x1(uint32_t taddr, const uint32_t *r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};"
                 :
                 : "r"(taddr), "r"(r[0]));
}
__device__ __forceinline__ void tmem_ld_x2(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_x2(uint32_t taddr, const uint32_t *r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};"
                 :
                 : "r"(taddr), "r"(r[0]), "r"(r[1]));
}
__device__ __forceinline__ void tmem_ld_x4(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_x4(uint32_t taddr, const uint32_t *r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};"
                 :
                 : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]));
}
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t *r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
                 :
                 : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]));
}
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t *r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
                 :
                 : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t *r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
                 :
                 : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]));
}

// N consecutive columns starting at taddr, split into power-of-two pieces,
// largest first (each piece starts at a multiple of its own width when taddr
// is a multiple of N's largest piece).
template <int N>
__device__ __forceinline__ void st_cols(uint32_t taddr, const uint32_t *r) {
    static_assert(N >= 1 && N <= 64, "columns");
    if constexpr (N >= 32) {
        tmem_st_x32(taddr, r);
        if constexpr (N > 32) st_cols<N - 32>(taddr + 32, r + 32);
    } else if constexpr (N >= 16) {
        tmem_st_x16(taddr, r);
        if constexpr (N > 16) st_cols<N - 16>(taddr + 16, r + 16);
    } else if constexpr (N >= 8) {
        tmem_st_x8(taddr, r);
        if constexpr (N > 8) st_cols<N - 8>(taddr + 8, r + 8);
    } else if constexpr (N >= 4) {
        tmem_st_x4(taddr, r);
        if constexpr (N > 4) st_cols<N - 4>(taddr + 4, r + 4);
    } else if constexpr (N >= 2) {
        tmem_st_x2(taddr, r);
        if constexpr (N > 2) st_cols<N - 2>(taddr + 2, r + 2);
    } else {
        tmem_st_x1(taddr, r);
    }
}
template <int N>
__device__ __forceinline__ void ld_cols(uint32_t taddr, uint32_t *r) {
    static_assert(N >= 1 && N <= 64, "columns");
    if constexpr (N >= 32) {
        tmem_ld_x32(taddr, r);
        if constexpr (N > 32) ld_cols<N - 32>(taddr + 32, r + 32);
    } else if constexpr (N >= 16) {
        tmem_ld_x16(taddr, r);
        if constexpr (N > 16) ld_cols<N - 16>(taddr + 16, r + 16);
    } else if constexpr (N >= 8) {
        tmem_ld_x8(taddr, r);
        if constexpr (N > 8) ld_cols<N - 8>(taddr + 8, r + 8);
    } else if constexpr (N >= 4) {
        tmem_ld_x4(taddr, r);
        if constexpr (N > 4) ld_cols<N - 4>(taddr + 4, r + 4);
    } else if constexpr (N >= 2) {
        tmem_ld_x2(taddr, r);
        if constexpr (N > 2) ld_cols<N - 2>(taddr + 2, r + 2);
    } else {
        tmem_ld_x1(taddr, r);
    }
}

// Wait for this thread's outstanding loads and make every later use of r[]
// depend on the wait.
template <int N>
__device__ __forceinline__ void wait_ld_bind(uint32_t *r) {
    wait_ld();
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// Float views.
template <int N>
__device__ __forceinline__ void store(uint32_t taddr, const float (&v)[N]) {
    uint32_t r[N];
#pragma unroll
    for (int i = 0; i < N; ++i) r[i] = __float_as_uint(v[i]);
    st_cols<N>(taddr, r);
}

}  // namespace tmem
}  // namespace bssm
