// Shared device helpers for the ArcLight B200 hot path (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "alb_cuda.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "arclight_b200 kernels are written for sm_100a only"
#endif

#define ALB_QK 32

// Return a status from a CUDA runtime call (host side).
#define ALB_CUDA_TRY(expr)                                                        \
    do {                                                                          \
        cudaError_t e__ = (expr);                                                 \
        if (e__ != cudaSuccess) { alb_set_last_cuda_error(e__, #expr); return ALB_ERR_CUDA; } \
    } while (0)

#define ALB_CHECK_ARG(cond)                                                       \
    do { if (!(cond)) { alb_set_last_error_msg("invalid argument: " #cond); return ALB_ERR_INVALID; } } while (0)

void alb_set_last_cuda_error(cudaError_t e, const char * what);
void alb_set_last_error_msg(const char * msg);
int  alb_sm_count();

// Programmatic dependent launch: the kernels below call these so that a
// dependent kernel (launched with cudaLaunchAttributeProgrammaticStreamSerialization)
// can start its prologue -- e.g. stream its weights -- while this grid drains.
__device__ __forceinline__ void alb_pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void alb_pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 16-byte read-only streaming load that does not allocate in L1.
__device__ __forceinline__ uint4 alb_ld_stream(const void * p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

__device__ __forceinline__ float alb_h2f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint16_t alb_f2h(float f) {
    return __half_as_ushort(__float2half_rn(f));
}

template <int W = 32>
__device__ __forceinline__ float alb_warp_sum(float v) {
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double alb_warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float alb_warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Launch helper: optionally marks the launch as a programmatic dependent of the
// previous kernel in the stream.
template <typename... KArgs, typename... Args>
static inline cudaError_t alb_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t stream, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------- mbarrier / bulk copy
__device__ __forceinline__ uint32_t alb_smem_addr(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void alb_mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(alb_smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void alb_mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void alb_mbar_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(alb_smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void alb_mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(alb_smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool alb_mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(alb_smem_addr(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Same, but the thread may be suspended (issuing nothing) until the phase
// completes or `hint_ns` elapses.
__device__ __forceinline__ bool alb_mbar_try_wait_sleep(uint64_t * bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(alb_smem_addr(bar)), "r"(parity), "r"(hint_ns) : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t alb_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait on an mbarrier phase: gives up after `ns` nanoseconds of
// %globaltimer (default 2 s) and returns false, so no wait can hang the GPU.
// Waiting threads sleep in the try_wait (at most 20 us per try) instead of
// spinning, so they take no issue slots from the warps that work.
__device__ __forceinline__ bool alb_mbar_wait(uint64_t * bar, uint32_t parity, uint64_t ns = 2000000000ull) {
    if (alb_mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = alb_globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (alb_mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if ((i & 15) == 0 && alb_globaltimer() - t0 > ns) return false;
    }
}
// Bounded wait that polls the phase with plain try_wait (no suspend-time hint),
// checking %globaltimer every 256 polls: for the short hand-offs of a
// streaming pipeline, where a waiter must resume the moment the phase flips.
__device__ __forceinline__ bool alb_mbar_wait_spin(uint64_t * bar, uint32_t parity, uint64_t ns = 2000000000ull) {
    if (alb_mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = alb_globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (alb_mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 0 && alb_globaltimer() - t0 > ns) return false;
    }
}
// Bounded wait for a thread with nothing else to do (a producer ahead of its
// consumers): polls with exponential __nanosleep backoff (32 ns .. 512 ns), so
// the waiting warp takes almost no issue slots from the warps that compute.
__device__ __forceinline__ bool alb_mbar_wait_backoff(uint64_t * bar, uint32_t parity, uint64_t ns = 2000000000ull) {
    if (alb_mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = alb_globaltimer();
    uint32_t nap = 32;
    for (;;) {
        __nanosleep(nap);
        if (alb_mbar_try_wait(bar, parity)) return true;
        if (nap < 512) nap <<= 1;
        if (alb_globaltimer() - t0 > ns) return false;
    }
}
// Bounded wait that naps between polls (__nanosleep, doubling from 32 ns up to
// max_nap ns): a waiting warp issues a handful of instructions per nap instead
// of polling back to back, leaving the issue slots to the warps that work.
// Gives up after `ns` nanoseconds of %globaltimer (default 2 s).
__device__ __forceinline__ bool alb_mbar_wait_nap(uint64_t * bar, uint32_t parity, uint32_t max_nap,
                                                  uint64_t ns = 2000000000ull) {
    if (alb_mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = alb_globaltimer();
    uint32_t nap = 32;
    for (;;) {
        __nanosleep(nap);
        if (alb_mbar_try_wait(bar, parity)) return true;
        if (nap < max_nap) nap <<= 1;
        if (alb_globaltimer() - t0 > ns) return false;
    }
}
// 1-D bulk copy global -> shared, completion counted on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void alb_bulk_g2s(void * dst_smem, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(alb_smem_addr(dst_smem)), "l"(src), "r"(bytes), "r"(alb_smem_addr(bar)) : "memory");
}

// ---------------------------------------------------------------- RMSNorm mean
// rms_norm_f32 (ops.cpp:703-710) sums the n fp32 squares in double in index
// order, then rounds sum / n to float.  A parallel sum of the same terms differs
// from that sequential sum by at most 2 (n - 1) u |sum| (u = 2^-53, recursive
// summation bound on each), so when both ends of [par - d, par + d] with
// d = 8 n u par give the same float mean, the sequential sum gives it too; only
// otherwise (probability ~ 16 n u / 2^-24 per norm) must the caller take the
// sequential sum itself.
__device__ __forceinline__ bool alb_rms_mean_certain(double par, int n) {
    const double d = par * (double)n * 0x1p-50;
    return (float)((par - d) / (double)n) == (float)((par + d) / (double)n);
}
// The same certificate without a division: inv_n is 1/n rounded to double,
// and the bounds are widened by par * 2^-48, which covers the rounding of
// inv_n, of par -/+ d and of the products.  When the float images of
// (par - d) * inv_n and (par + d) * inv_n agree, the reference's float mean
// (its sequential sum divided by n, rounded to double, then to float) is that
// value, returned in `mean`; otherwise the caller takes the sequential sum.
__device__ __forceinline__ bool alb_rms_mean_cert(double par, int n, double inv_n, float & mean) {
    const double d = par * (double)n * 0x1p-50 + par * 0x1p-48;
    const float lo = (float)((par - d) * inv_n), hi = (float)((par + d) * inv_n);
    mean = lo;
    return lo == hi;
}
// Pairwise sum of v[0..N) (a fixed tree: depth log2 N instead of a chain of N).
template <int N>
__device__ __forceinline__ double alb_tree_sum(const double * v) {
    if constexpr (N == 1) return v[0];
    else return alb_tree_sum<N / 2>(v) + alb_tree_sum<N - N / 2>(v + N / 2);
}
// The sequential sum of the squares of x[0..n) (one thread).
__device__ __forceinline__ double alb_rms_seq_sum(const float * x, int n) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += (double)__fmul_rn(x[i], x[i]);
    return s;
}

// ---------------------------------------------------------------- reference expf / silu
// nnml_v_expf (arm.cpp:1757-1787) per lane, so SwiGLU matches the reference's
// NEON path bit for bit: exp(x) = 2^n (1 + p(b)), n from the 1.5*2^23 shift,
// b = x - n ln2 (two-part ln2), degree-5 polynomial; |n| > 126 / > 192 use the
// scaled / saturated forms.  Same algorithm, restated with explicit roundings.
__device__ __forceinline__ float alb_ref_expf(float x) {
    const float r = 0x1.8p23f;
    const float z = __fmaf_rn(x, 0x1.715476p+0f, r);
    const float n = __fsub_rn(z, r);
    const float b = __fmaf_rn(-n, 0x1.7f7d1cp-20f, __fmaf_rn(-n, 0x1.62e4p-1f, x));
    const uint32_t e = __float_as_uint(z) << 23;
    const float k = __uint_as_float(e + 0x3f800000u);
    const float u = __fmul_rn(b, b);
    const float j = __fmaf_rn(__fmaf_rn(__fmaf_rn(0x1.0e4020p-7f, b, 0x1.573e2ep-5f), u,
                                        __fmaf_rn(0x1.555e66p-3f, b, 0x1.fffdb6p-2f)),
                              u, __fmul_rn(0x1.ffffecp-1f, b));
    const float an = fabsf(n);
    if (!(an > 126.0f)) return __fmaf_rn(j, k, k);
    const uint32_t d = (n <= 0.0f) ? 0x82000000u : 0u;
    const float s1 = __uint_as_float(d + 0x7f000000u);
    const float s2 = __uint_as_float(e - d);
    if (an > 192.0f) return __fmul_rn(s1, s1);
    return __fmul_rn(__fmaf_rn(s2, j, s2), s1);
}
// nnml_vec_swiglu_f32 NEON path (arm.cpp:1789-1809): (x / (1 + exp(0 - x))) * g
__device__ __forceinline__ float alb_swiglu1(float x, float g) {
    return __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, alb_ref_expf(__fsub_rn(0.0f, x)))), g);
}
