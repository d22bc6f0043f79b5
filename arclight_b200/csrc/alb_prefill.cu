// Prefill Q4_0 x Q8_0 mat-mul on the sm_100a tensor cores (tcgen05.mma
// kind::i8, accumulators in TMEM).
//
// Y[m][n] = fp32 fma chain over the blocks b in order of
// float(I(m,n,b)) * (dx[m][b] * dw[n][b]), I = sum over the 32 values of block
// b of q8[m][k] * (q4[n][k] - 8): the arithmetic of the reference's
// nnml_gemm_q4_0_4x4_q8_0 (gemm.cpp:495-974: scvtf #4 of 16 I, fmul of the two
// scales, fmla into the row's accumulator, block after block), which is the
// mat-vec's chain, so every output row is bit-identical to the mat-vec of that
// row.  Because the scales change every 32 values of K, every block is one MMA
// (M = 128 tokens, N = 64 rows of W, K = 32) into a fresh TMEM accumulator,
// and the epilogue warps read it back (tcgen05.ld) and advance their fp32
// chains while the tensor core computes the next block into the other half of
// the TMEM allocation.
//
// Operands in shared memory, K-major without swizzle (core matrices of 8 rows
// x 16 bytes; the two 16-byte halves of a block are the two K chunks):
//   A: the 128 token rows' int8 Q8_0 values of block b (4 KiB)
//   B: the 64 weight rows' nibbles of block b unpacked to int8 q - 8 (2 KiB)
// Every wait is bounded (2 s); on a timeout the kernel records an error code,
// waits (bounded) for its MMAs in flight, frees its TMEM and returns.
#include "alb_common.cuh"
#include "alb_internal.h"
#include "alb_q4_dev.cuh"

namespace alb {

static constexpr int PG_M = 128;          // tokens per tile (TMEM lanes)
static constexpr int PG_N = 64;           // weight rows per tile (TMEM columns per buffer)
static constexpr int PG_THREADS = 256;    // 8 warps: all load, thread 0 issues, all read back
static constexpr uint32_t PG_TMEM_COLS = 2 * PG_N;

static constexpr int PG_STAGES = 4;       // cp.async ring depth (blocks of K in flight)

struct PgShared {
    alignas(128) int8_t a[PG_STAGES][PG_M * 32];   // MMA operand A per stage (core-matrix layout)
    alignas(128) int8_t b[2][PG_N * 32];           // MMA operand B (unpacked) for blocks b & 1
    alignas(16) uint8_t nib[PG_STAGES][PG_N * 16]; // W nibbles as loaded
    alignas(16) float dx[PG_STAGES][PG_M];         // activation block scales (fp16-rounded)
    alignas(16) uint32_t dww[PG_STAGES][PG_N];     // 4-byte words holding the weight block scale
    alignas(16) float dwf[2][PG_N];                // weight block scale as fp32
    uint64_t mma_done[2];
    uint32_t tmem_base;
    int abort_flag;
};

__device__ __forceinline__ uint32_t pg_smem(const void * p) { return alb_smem_addr(p); }

// K-major, no swizzle: core matrix = 8 rows x 16 B contiguous; K chunk stride
// (leading byte offset) 128 B, 8-row group stride (stride byte offset) 256 B.
__device__ __forceinline__ uint64_t pg_desc(const void * smem) {
    const uint64_t addr = pg_smem(smem);
    return ((addr >> 4) & 0x3FFFull) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
           (1ull << 46);   // descriptor version 1 (sm_100); base offset 0, layout SWIZZLE_NONE
}

// instruction descriptor: D s32, A s8, B s8, both K-major, N = 64, M = 128
static constexpr uint32_t PG_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PG_N >> 3) << 17) |
                                     ((uint32_t)(PG_M >> 4) << 24);

// byte offset of (row r, 16-byte chunk c) in a K-major core-matrix tile
__device__ __forceinline__ int pg_off(int r, int c) { return (r >> 3) * 256 + c * 128 + (r & 7) * 16; }

__device__ __forceinline__ void pg_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void pg_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Activations of the GEMM: xq int8 [M][K] row-major, xd float [M][K/32]
// (fp16-rounded Q8_0 scale), from fp32 rows (one warp per 32-value block,
// quantize_row_q8_0 semantics, arm.cpp:1819-1853).
__global__ void k_pg_quant(const float * __restrict__ x, int64_t M, int64_t K, int8_t * __restrict__ xq,
                           float * __restrict__ xd) {
    alb_pdl_wait();
    const int lane = threadIdx.x & 31;
    const int64_t nb = K / 32;
    const int64_t w = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (w >= M * nb) return;
    const int64_t m = w / nb, b = w - m * nb;
    const float v = x[m * K + b * 32 + lane];
    int8_t q;
    uint16_t dh;
    q8_block_lane(v, q, dh);
    xq[m * K + b * 32 + lane] = q;
    if (lane == 0) xd[m * nb + b] = alb_h2f(dh);
}

// Same from block_q8_0 rows (the reference layout, nnml.h:695-700).
__global__ void k_pg_from_q8(const uint8_t * __restrict__ src, int64_t M, int64_t K, int8_t * __restrict__ xq,
                             float * __restrict__ xd) {
    alb_pdl_wait();
    const int64_t nb = K / 32;
    const int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= M * nb) return;
    const uint8_t * s = src + blk * 34;
    const uint16_t dh = (uint16_t)(s[0] | (s[1] << 8));
    xd[blk] = alb_h2f(dh);
    int8_t * d = xq + blk * 32;   // row-major [M][K]: block blk = m * nb + b lands at m*K + 32 b
    for (int j = 0; j < 32; ++j) d[j] = (int8_t)s[2 + j];
}

__device__ __forceinline__ bool pg_wait(PgShared & sh, int buf, uint32_t parity, int * err) {
    if (alb_mbar_wait(&sh.mma_done[buf], parity)) return true;
    if ((threadIdx.x & 31) == 0) atomicExch(err, ALB_DEVERR_MBAR_TIMEOUT);
    sh.abort_flag = 1;
    return false;
}

template <int OUT>   // 0: y = acc (+ residual), 1: SwiGLU of interleaved (gate, up) rows
__global__ void __launch_bounds__(PG_THREADS, 2)
k_prefill_gemm(const uint8_t * __restrict__ Wn, const uint8_t * __restrict__ Ws, int64_t N, int64_t K,
               const int8_t * __restrict__ xq, const float * __restrict__ xd, int64_t M, float * __restrict__ y,
               int64_t y_stride, const float * __restrict__ residual, int * err) {
    __shared__ PgShared sh;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t n0 = (int64_t)blockIdx.x * PG_N, m0 = (int64_t)blockIdx.y * PG_M;
    const int64_t nb = K / 32, rb = q4_row_bytes(K);   // row-interleaved layout: nibbles at 0, scales at K/2
    if (tid == 0) {
        alb_mbar_init(&sh.mma_done[0], 1);
        alb_mbar_init(&sh.mma_done[1], 1);
        sh.abort_flag = 0;
        alb_mbar_fence_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(pg_smem(&sh.tmem_base)), "r"(PG_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pg_fence_before();
    __syncthreads();
    pg_fence_after();
    const uint32_t tmem = sh.tmem_base;
    alb_pdl_wait();

    // epilogue mapping: warp w reads TMEM lanes 32*(w%4).., columns 32*(w/4)..
    const int quarter = warp & 3, chalf = warp >> 2;
    const int row = quarter * 32 + lane;                 // token row within the tile
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
    uint32_t issued = 0, waited = 0;                     // MMAs committed / completions consumed (per buffer parity)

    // cp.async of block kb's inputs into ring stage kb % PG_STAGES (zero-filled past M / N)
    auto prefetch = [&](int64_t kb) {
        const int st = (int)(kb % PG_STAGES);
        if (kb < nb) {
            {   // A: thread t -> row t/2, chunk t%2 (16 B)
                const int r = tid >> 1, c = tid & 1;
                const bool in = m0 + r < M;
                const int8_t * src = xq + (in ? (m0 + r) * K + kb * 32 + c * 16 : 0);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                             :: "r"(pg_smem(sh.a[st] + pg_off(r, c))), "l"(src), "r"(in ? 16 : 0) : "memory");
            }
            if (tid < PG_N) {
                const bool in = n0 + tid < N;
                const uint8_t * src = Wn + (in ? (n0 + tid) * rb + kb * 16 : 0);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                             :: "r"(pg_smem(sh.nib[st] + tid * 16)), "l"(src), "r"(in ? 16 : 0) : "memory");
            } else if (tid < 2 * PG_N) {
                const int n = tid - PG_N;
                const bool in = n0 + n < N;
                const uint8_t * src = Ws + (in ? ((n0 + n) * rb + ((kb * 2) & ~(int64_t)3)) : 0);
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;"
                             :: "r"(pg_smem(&sh.dww[st][n])), "l"(src), "r"(in ? 4 : 0) : "memory");
            } else {
                const int r = tid - 2 * PG_N;
                const bool in = m0 + r < M;
                const float * src = xd + (in ? (m0 + r) * nb + kb : 0);
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;"
                             :: "r"(pg_smem(&sh.dx[st][r])), "l"(src), "r"(in ? 4 : 0) : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");   // one group per block (empty past the end)
    };

    // dxr: this thread's token-row scale of block kb, read from the ring when the
    // block landed (the ring stage is refilled by other warps while this one may
    // still be in its epilogue, so the scale is carried in a register)
    auto epilogue = [&](int64_t kb, float dxr) {
        const int s = (int)(kb & 1);
        pg_fence_after();
        uint32_t c[32];
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(s * PG_N + chalf * 32);
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                     "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                     "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                     : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3]), "=r"(c[4]), "=r"(c[5]), "=r"(c[6]), "=r"(c[7]),
                       "=r"(c[8]), "=r"(c[9]), "=r"(c[10]), "=r"(c[11]), "=r"(c[12]), "=r"(c[13]), "=r"(c[14]),
                       "=r"(c[15]), "=r"(c[16]), "=r"(c[17]), "=r"(c[18]), "=r"(c[19]), "=r"(c[20]), "=r"(c[21]),
                       "=r"(c[22]), "=r"(c[23]), "=r"(c[24]), "=r"(c[25]), "=r"(c[26]), "=r"(c[27]), "=r"(c[28]),
                       "=r"(c[29]), "=r"(c[30]), "=r"(c[31])
                     : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const float * dw = sh.dwf[s] + chalf * 32;
        // float(I) exactly as 2^23 * 1.5 + I - 2^23 * 1.5 (|I| < 2^22): integer add +
        // fp32 subtract instead of a conversion; dx * dw is exact (11 x 11 bits)
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float t = __fsub_rn(__int_as_float((int)c[j] + 0x4B400000), 12582912.0f);
            acc[j] = __fmaf_rn(t, __fmul_rn(dxr, dw[j]), acc[j]);
        }
        pg_fence_before();
    };

    for (int64_t kb = 0; kb < PG_STAGES - 1; ++kb) prefetch(kb);
    bool ok = true;
    float dx_prev = 0.0f, dx_cur = 0.0f;   // this row's activation scales of blocks b-1 and b
    for (int64_t b = 0; b < nb && ok; ++b) {
        const int s = (int)(b & 1), st = (int)(b % PG_STAGES);
        asm volatile("cp.async.wait_group %0;" :: "n"(PG_STAGES - 2) : "memory");   // block b has landed
        __syncthreads();
        dx_prev = dx_cur;
        dx_cur = sh.dx[st][row];   // stage st is refilled only after the next iteration's epilogue
        if (tid >= PG_N && tid < 2 * PG_N) {   // weight scales of block b, once per block
            const int n = tid - PG_N;
            const uint32_t wd = sh.dww[st][n];
            sh.dwf[s][n] = alb_h2f((uint16_t)((b & 1) ? (wd >> 16) : (wd & 0xFFFFu)));
        }
        if (tid < PG_N) {   // B: 16 nibble bytes of row tid -> 2 chunks of int8 (q - 8)
            const uint4 w = *reinterpret_cast<const uint4 *>(sh.nib[st] + tid * 16);
            const uint4 lo = make_uint4(__vsub4(w.x & 0x0F0F0F0Fu, 0x08080808u), __vsub4(w.y & 0x0F0F0F0Fu, 0x08080808u),
                                        __vsub4(w.z & 0x0F0F0F0Fu, 0x08080808u), __vsub4(w.w & 0x0F0F0F0Fu, 0x08080808u));
            const uint4 hi = make_uint4(__vsub4((w.x >> 4) & 0x0F0F0F0Fu, 0x08080808u),
                                        __vsub4((w.y >> 4) & 0x0F0F0F0Fu, 0x08080808u),
                                        __vsub4((w.z >> 4) & 0x0F0F0F0Fu, 0x08080808u),
                                        __vsub4((w.w >> 4) & 0x0F0F0F0Fu, 0x08080808u));
            *reinterpret_cast<uint4 *>(sh.b[s] + pg_off(tid, 0)) = lo;
            *reinterpret_cast<uint4 *>(sh.b[s] + pg_off(tid, 1)) = hi;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic / cp.async stores -> tensor core
        __syncthreads();
        if (tid == 0) {
            pg_fence_after();
            const uint64_t da = pg_desc(sh.a[st]), db = pg_desc(sh.b[s]);
            const uint32_t zero = 0;
            asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                         "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
                         :: "r"(tmem + (uint32_t)(s * PG_N)), "l"(da), "l"(db), "r"(PG_IDESC), "r"(zero), "r"(zero)
                         : "memory");
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         :: "r"(pg_smem(&sh.mma_done[s])) : "memory");
        }
        ++issued;
        if (b > 0) {   // block b-1 (other TMEM buffer) while the tensor core works on block b
            ok = pg_wait(sh, s ^ 1, (uint32_t)(((b - 1) >> 1) & 1), err);
            if (ok) { epilogue(b - 1, dx_prev); ++waited; }
        }
        // block b-1 is consumed (MMA done, scales read): its ring stage takes block b + PG_STAGES - 1
        prefetch(b + PG_STAGES - 1);
        __syncthreads();
        if (sh.abort_flag) ok = false;
    }
    if (ok) {
        const int64_t b = nb - 1;
        ok = pg_wait(sh, (int)(b & 1), (uint32_t)((b >> 1) & 1), err);
        if (ok) { epilogue(b, dx_cur); ++waited; }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");   // no copy in flight past this point
    if (!ok) {
        // every committed MMA must have completed before the TMEM is freed
        for (uint32_t q = waited; q < issued; ++q) {
            const int64_t b = q;
            alb_mbar_wait(&sh.mma_done[b & 1], (uint32_t)((b >> 1) & 1));
        }
    }
    pg_fence_before();
    __syncthreads();
    if (warp == 0) {
        pg_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(PG_TMEM_COLS) : "memory");
    }
    if (!ok) return;
    const int64_t m = m0 + row;
    if (m >= M) return;
    const int64_t nbase = n0 + chalf * 32;
    if constexpr (OUT == 0) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int64_t n = nbase + j;
            if (n < N) {
                const float v = acc[j];
                y[m * y_stride + n] = residual ? __fadd_rn(v, residual[m * y_stride + n]) : v;
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int64_t n = nbase + 2 * j;
            if (n + 1 < N)
                y[m * y_stride + n / 2] = alb_swiglu1(acc[2 * j], acc[2 * j + 1]);
        }
    }
}

size_t prefill_ws_bytes(int64_t M, int64_t K) {
    const size_t q = ((size_t)M * K + 255) & ~(size_t)255;
    return q + (size_t)M * (K / 32) * 4;
}

// x fp32 [M][K] (already normalized if needed) -> y: workspace prefill_ws_bytes(M, K)
cudaError_t launch_prefill_gemm(const uint8_t * W, int64_t N, int64_t K, const float * x, const void * xq_blocks,
                                int64_t M, float * y, int64_t y_stride, const float * residual, bool swiglu, void * ws,
                                int * err, bool pdl, cudaStream_t st) {
    int8_t * xq = reinterpret_cast<int8_t *>(ws);
    float * xd = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(ws) + (((size_t)M * K + 255) & ~(size_t)255));
    const int64_t nblk = M * (K / 32);
    cudaError_t e;
    if (x) e = alb_launch(k_pg_quant, dim3((unsigned)((nblk + 7) / 8)), dim3(256), 0, st, pdl, x, M, K, xq, xd);
    else e = alb_launch(k_pg_from_q8, dim3((unsigned)((nblk + 255) / 256)), dim3(256), 0, st, pdl,
                        reinterpret_cast<const uint8_t *>(xq_blocks), M, K, xq, xd);
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)((N + PG_N - 1) / PG_N), (unsigned)((M + PG_M - 1) / PG_M));
    const uint8_t * Ws = W + K / 2;   // scales of row n at Ws + n * q4_row_bytes(K)
    if (swiglu)
        return alb_launch(k_prefill_gemm<1>, grid, dim3(PG_THREADS), 0, st, pdl, W, Ws, N, K, (const int8_t *)xq,
                          (const float *)xd, M, y, y_stride, residual, err);
    return alb_launch(k_prefill_gemm<0>, grid, dim3(PG_THREADS), 0, st, pdl, W, Ws, N, K, (const int8_t *)xq,
                      (const float *)xd, M, y, y_stride, residual, err);
}

}  // namespace alb

using namespace alb;

extern "C" size_t alb_gemm_workspace_bytes(int64_t M, int64_t K) {
    if (M <= 0 || K <= 0 || K % 32) return 0;
    return prefill_ws_bytes(M, K);
}

extern "C" int alb_gemm_q4_0_q8_0(const void * W, const void * xq, float * y, int64_t M, int64_t N, int64_t K,
                                  const float * residual, void * workspace, void * stream) {
    ALB_CHECK_ARG(W && xq && y && workspace && M > 0 && N > 0 && K > 0 && K % 32 == 0);
    ALB_CHECK_ARG(M < ((int64_t)1 << 24) && N < ((int64_t)1 << 30) && K <= 65536);
    ALB_CUDA_TRY(launch_prefill_gemm((const uint8_t *)W, N, K, nullptr, xq, M, y, N, residual, false, workspace,
                                     device_error_ptr(), true, (cudaStream_t)stream));
    return ALB_OK;
}
