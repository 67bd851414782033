// bssm_check.cu -- one-pass input checks for the Python API.
//
// bayesian_layer validates its inputs before any recurrence runs
// (catid/bayes-ssm bayes_ssm/bayesian_layer.py:105-128): every tensor must be
// finite, process variances nonnegative, observation variances strictly
// positive.  Done with torch ops, each check is several elementwise kernels
// and a reduction over a full-size temporary (and a BF16 input is first
// widened to FP32).  This kernel reads a tensor once, in its own dtype, and
// ORs three flags into one device word; the caller reads the word back and
// raises the reference's error for the first failing check.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "bayes_ssm_b200.h"
#include "bssm_flags.cuh"
#include "bssm_internal.h"

namespace bssm {
namespace {

__device__ __forceinline__ float widen(float x) { return x; }
__device__ __forceinline__ float widen(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float widen(__half x) { return __half2float(x); }

// Grid-stride over 16-byte chunks (when the base is 16-byte aligned), then
// the ragged tail element by element.
template <typename T>
__global__ void check_values_kernel(const T *__restrict__ x, long n, unsigned *flags) {
    constexpr int EC = 16 / static_cast<int>(sizeof(T));
    unsigned f = 0;
    const long tid = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long nthreads = static_cast<long>(gridDim.x) * blockDim.x;
    long done = 0;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const long nvec = n / EC;
        const uint4 *xv = reinterpret_cast<const uint4 *>(x);
        // four independent 16-byte loads in flight per thread, then the rest
        long i = tid;
        for (; i + 3 * nthreads < nvec; i += 4 * nthreads) {
            uint4 w[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) w[u] = __ldg(xv + i + u * nthreads);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const T *e = reinterpret_cast<const T *>(&w[u]);
#pragma unroll
                for (int j = 0; j < EC; ++j) f |= check_flags_of(widen(e[j]));
            }
        }
        for (; i < nvec; i += nthreads) {
            const uint4 w = __ldg(xv + i);
            const T *e = reinterpret_cast<const T *>(&w);
#pragma unroll
            for (int j = 0; j < EC; ++j) f |= check_flags_of(widen(e[j]));
        }
        done = nvec * EC;
    }
    for (long i = done + tid; i < n; i += nthreads) f |= check_flags_of(widen(x[i]));
    f = __reduce_or_sync(0xffffffffu, f);
    if ((threadIdx.x & 31) == 0 && f != 0) atomicOr(flags, f);
}

template <typename T>
int launch_check(const void *x, long n, unsigned *flags, cudaStream_t st) {
    constexpr int threads = 256;
    const long work = (n + 16 / static_cast<long>(sizeof(T)) - 1) / (16 / static_cast<long>(sizeof(T)));
    long blocks = (work + threads - 1) / threads;
    if (blocks > 148L * 8) blocks = 148L * 8;
    if (blocks < 1) blocks = 1;
    check_values_kernel<T><<<static_cast<unsigned>(blocks), threads, 0, st>>>(static_cast<const T *>(x), n, flags);
    return check_launch("check_values");
}

}  // namespace
}  // namespace bssm

extern "C" int bssm_check_values(const void *x, long n, int dtype, unsigned *flags, void *stream) {
    using namespace bssm;
    if (n < 0 || flags == nullptr || (n > 0 && x == nullptr)) return fail(BSSM_ERR_INVALID, "check_values: bad arguments");
    if (n == 0) return BSSM_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (dtype) {
        case BSSM_F32: return launch_check<float>(x, n, flags, st);
        case BSSM_BF16: return launch_check<__nv_bfloat16>(x, n, flags, st);
        case BSSM_F16: return launch_check<__half>(x, n, flags, st);
    }
    return fail(BSSM_ERR_UNSUPPORTED, "check_values: dtype %d", dtype);
}

// ---------------------------------------------------------------------------
// FP32 FMA throughput probe: the denominator of the recurrence kernels' FP32
// roofline, measured on the GPU at hand rather than taken from a datasheet.
// Every thread runs kChains independent FMA chains (enough instructions in
// flight to hide the FMA latency on every sub-partition); the result is
// stored only under a condition the values never meet, so no FMA is dead.
namespace bssm {
namespace {
constexpr int kProbeChains = 8;
__global__ void __launch_bounds__(256) fma_probe_kernel(float *out, int iters, float a, float b) {
    float x[kProbeChains];
#pragma unroll
    for (int c = 0; c < kProbeChains; ++c) x[c] = static_cast<float>(threadIdx.x + c) * 1e-3f;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
            for (int c = 0; c < kProbeChains; ++c) x[c] = fmaf(x[c], a, b);
    }
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < kProbeChains; ++c) s += x[c];
    if (s == 1234.5678f) out[blockIdx.x * blockDim.x + threadIdx.x] = s;
}
}  // namespace
}  // namespace bssm

extern "C" long bssm_debug_fma_probe_flops(int blocks, int iters) {
    return 2L * blocks * 256 * bssm::kProbeChains * 8 * iters;
}

extern "C" int bssm_debug_fma_probe(float *out, int blocks, int iters, void *stream) {
    using namespace bssm;
    if (blocks < 1 || iters < 1 || out == nullptr) return fail(BSSM_ERR_INVALID, "fma probe: bad arguments");
    // a * x + b with |a| < 1 stays bounded: no overflow, no denormal slow path
    fma_probe_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(out, iters, 0.999f, 1e-3f);
    return check_launch("fma probe");
}
