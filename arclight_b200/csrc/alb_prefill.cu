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
// chains while the tensor core computes the next blocks into the other
// buffers of the TMEM allocation.
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
static constexpr int PG_D = 5;            // operand ring stages (blocks of K in flight)
static constexpr int PG_LAG = 2;          // blocks the loader keeps in flight before publishing one
static constexpr int PG_NB = 4;           // TMEM accumulator buffers (blocks the MMA may run ahead)
static constexpr int PG_NI = PG_NB;       // unpack + MMA-issue warps (issuer i: blocks i, i + PG_NI, .., TMEM buffer i)
static constexpr int PG_EW = 4 * (PG_N / 32);   // epilogue warps: 4 TMEM lane quarters x 32-column groups
static constexpr int PG_E0 = 1 + PG_NI;   // first epilogue warp
static constexpr int PG_THREADS = (1 + PG_NI + PG_EW) * 32;   // warp 0 loads, 1..PG_NI issue, then the epilogue
static constexpr uint32_t PG_TMEM_COLS = PG_NB * PG_N;
static constexpr int PG_CTAS = 512 / PG_TMEM_COLS;   // CTAs per SM (the SM's 512 TMEM columns)

struct PgShared {
    alignas(128) int8_t a[PG_D][PG_M * 32];   // MMA operand A per stage (core-matrix layout)
    alignas(128) int8_t b[PG_D][PG_N * 32];   // MMA operand B (nibbles unpacked to int8 q - 8) per stage
    alignas(16) uint8_t nib[PG_D][PG_N * 16]; // W nibbles as loaded
    alignas(16) float dx[PG_D][PG_M];         // activation block scales (fp16-rounded)
    alignas(16) uint16_t dws[2][PG_N][8];     // weight scales of blocks 8j .. 8j+7 (slot j % 2), one 16-byte load per row
    alignas(16) float dwf[PG_D][PG_N];        // weight block scale as fp32
    uint64_t full[PG_D];                      // stage loaded and fenced for the tensor core (loader lane 0)
    uint64_t empty[PG_D];                     // stage consumed (its MMA + the epilogue warps' scale reads)
    uint64_t tfull[PG_NB];                    // accumulator ready (MMA commit + the issuer's dwf release)
    uint64_t tempty[PG_NB];                   // accumulator read back (epilogue warps)
    uint64_t drain;                           // every MMA of the CTA complete (one commit per issuer)
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

// 16 TMEM columns of this warp's 32 lanes <- v (two 8-column tcgen05.st: a
// store takes a run of consecutive registers, so narrow ones keep the
// epilogue within its register budget; the caller waits with wait::st).
__device__ __forceinline__ void pg_tmem_fill16(uint32_t taddr, uint32_t v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" :: "r"(taddr), "r"(v) : "memory");
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" :: "r"(taddr + 8u), "r"(v) : "memory");
}
// float(I) from the accumulator: every buffer is pre-set to bits(1.5 * 2^23)
// before its MMA accumulates the int32 block dot onto it, so the accumulator
// holds bits(1.5 * 2^23) + I and one fp32 subtract gives float(I) exactly
// (|I| < 2^22).
static constexpr uint32_t PG_BIAS = 0x4B400000u;

__device__ __forceinline__ void pg_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void pg_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Activations of the GEMM: xq int8 [M][K] row-major, xd float [K/32][Mp]
// (block-major, Mp = M rounded up to 4: one block's scales of 128 tokens are
// one contiguous 512-byte run) holding the fp16-rounded Q8_0 scales, from fp32
// rows (one warp per 32-value block, quantize_row_q8_0 semantics,
// arm.cpp:1819-1853).
__host__ __device__ inline int64_t pg_mpad(int64_t M) { return (M + 3) & ~(int64_t)3; }

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
    if (lane == 0) xd[b * pg_mpad(M) + m] = alb_h2f(dh);
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
    xd[(blk % nb) * pg_mpad(M) + blk / nb] = alb_h2f(dh);
    int8_t * d = xq + blk * 32;   // row-major [M][K]: block blk = m * nb + b lands at m*K + 32 b
    for (int j = 0; j < 32; ++j) d[j] = (int8_t)s[2 + j];
}

// Bounded wait on one of the kernel's mbarriers; a timeout records an error
// code and raises the CTA's abort flag (every role then leaves its loop).
__device__ __forceinline__ bool pg_wait(PgShared & sh, uint64_t * bar, uint32_t parity, int * err) {
    if (alb_mbar_wait(bar, parity)) return true;
    atomicExch(err, ALB_DEVERR_MBAR_TIMEOUT);
    sh.abort_flag = 1;
    return false;
}
__device__ __forceinline__ bool pg_aborted(PgShared & sh) { return *reinterpret_cast<volatile int *>(&sh.abort_flag) != 0; }

// Warp-specialised pipeline, one CTA per (64 weight rows, 128 tokens), two CTAs
// per SM:
//   warp 0      loads block b's operands into ring stage b % PG_D (cp.async)
//               once empty[stage] says the stage's previous block is consumed;
//               PG_LAG blocks later its lanes wait for those copies, fence them
//               for the async proxy (the tensor core reads A) and lane 0
//               publishes the stage on full[stage];
//   warps 1..4  (issuer i: blocks i, i + 4, ..; TMEM buffer i) unpack the
//               nibbles into the B operand, convert the weight scales, and
//               (lane 0) issue the block's MMA once tempty[i] says the buffer's
//               previous block was read back; the MMA's commit arrives on
//               tfull[i] and empty[stage].  One issuer's serial path (waits,
//               unpack, proxy fence, issue) is ~1.2 us per block: four of them
//               keep the tensor core and the epilogue fed;
//   warps 5..12 pre-set every buffer to the float-conversion bias, read each
//               block's accumulator back (tcgen05.ld: warp w reads TMEM lanes
//               32 (w % 4) .., columns 32 ((w - 5) / 4) ..), set the bias again,
//               release the buffer, advance their 32 fp32 chains, release the
//               stage.
// No CTA-wide barrier per block: the tensor core runs up to PG_NB blocks ahead
// of the epilogue and the loads PG_D blocks ahead of the tensor core.
template <int OUT>   // 0: y = acc (+ residual), 1: SwiGLU of interleaved (gate, up) rows
__global__ void __launch_bounds__(PG_THREADS, PG_CTAS)
k_prefill_gemm(const uint8_t * __restrict__ Wn, const uint8_t * __restrict__ Ws, int64_t N, int64_t K,
               const int8_t * __restrict__ xq, const float * __restrict__ xd, int64_t M, float * __restrict__ y,
               int64_t y_stride, const float * __restrict__ residual, int * err) {
    extern __shared__ __align__(128) uint8_t pg_dyn[];
    PgShared & sh = *reinterpret_cast<PgShared *>(pg_dyn);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t n0 = (int64_t)blockIdx.x * PG_N, m0 = (int64_t)blockIdx.y * PG_M;
    const int64_t nb = K / 32, rb = q4_row_bytes(K);   // row-interleaved layout: nibbles at 0, scales at K/2
    const int64_t Mp = pg_mpad(M);                       // row stride of the block-major activation scales
    if (tid == 0) {
        for (int i = 0; i < PG_D; ++i) { alb_mbar_init(&sh.full[i], 1); alb_mbar_init(&sh.empty[i], 1 + PG_EW); }
        for (int i = 0; i < PG_NB; ++i) { alb_mbar_init(&sh.tfull[i], 2); alb_mbar_init(&sh.tempty[i], PG_EW); }
        alb_mbar_init(&sh.drain, PG_NI);
        sh.abort_flag = 0;
        alb_mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(pg_smem(&sh.tmem_base)), "r"(PG_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    pg_fence_before();
    __syncthreads();
    pg_fence_after();
    const uint32_t tmem = sh.tmem_base;
    alb_pdl_wait();

    const int quarter = warp & 3, chalf = (warp - PG_E0) >> 2;   // epilogue warps: lane quarter, 32-column group
    const int row = quarter * 32 + lane;                     // token row within the tile
    float acc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = 0.0f;

    if (warp == 0) {
        // ------------------------------------------------------------ loads
        int64_t published = 0;   // blocks published on full[]
        for (int64_t b = 0; b < nb; ++b) {
            const int st = (int)(b % PG_D);
            if (b >= PG_D && !pg_wait(sh, &sh.empty[st], (uint32_t)((b / PG_D - 1) & 1), err)) break;
            if (pg_aborted(sh)) break;
            for (int i = lane; i < PG_M * 2; i += 32) {   // A: row i/2, 16-byte chunk i%2
                const int r = i >> 1, c = i & 1;
                const bool in = m0 + r < M;
                const int8_t * src = xq + (in ? (m0 + r) * K + b * 32 + c * 16 : 0);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                             :: "r"(pg_smem(sh.a[st] + pg_off(r, c))), "l"(src), "r"(in ? 16 : 0) : "memory");
            }
#pragma unroll
            for (int k = 0; k < PG_N / 32; ++k) {        // nibbles of rows lane, lane + 32 (and every 8 blocks their scales)
                const int n = lane + 32 * k;
                const bool in = n0 + n < N;
                const uint8_t * srcn = Wn + (in ? (n0 + n) * rb + b * 16 : 0);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                             :: "r"(pg_smem(sh.nib[st] + n * 16)), "l"(srcn), "r"(in ? 16 : 0) : "memory");
                if ((b & 7) == 0) {   // scales of blocks b .. b+7 (16 bytes, zero past the row's last block)
                    const int64_t nbytes = (nb - b) * 2 < 16 ? (nb - b) * 2 : 16;
                    const uint8_t * srcs = Ws + (in ? (n0 + n) * rb + b * 2 : 0);
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                                 :: "r"(pg_smem(sh.dws[(b >> 3) & 1][n])), "l"(srcs), "r"(in ? (int)nbytes : 0) : "memory");
                }
            }
            {   // activation scales of the 128 rows: one contiguous run of the block-major xd
                const int r = 4 * lane;
                const int64_t left = M - (m0 + r);
                const int bytes = left >= 4 ? 16 : left > 0 ? (int)left * 4 : 0;
                const float * src = xd + (bytes ? b * Mp + m0 + r : 0);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                             :: "r"(pg_smem(&sh.dx[st][r])), "l"(src), "r"(bytes) : "memory");
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            if (b >= PG_LAG) {   // block b - PG_LAG has landed: fence it for the tensor core, publish it
                asm volatile("cp.async.wait_group %0;" :: "n"(PG_LAG) : "memory");
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) alb_mbar_arrive(&sh.full[(int)((b - PG_LAG) % PG_D)]);
            }
            published = b - PG_LAG + 1;
        }
        asm volatile("cp.async.wait_all;" ::: "memory");   // no copy in flight past this point
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (!pg_aborted(sh) && lane == 0)
            for (int64_t j = published < 0 ? 0 : published; j < nb; ++j) alb_mbar_arrive(&sh.full[(int)(j % PG_D)]);
    } else if (warp < PG_E0) {
        // ------------------------------------------- unpack + MMA issue
        const int tb = warp - 1;   // this issuer's TMEM buffer; its blocks are tb, tb + PG_NI, ..
        for (int64_t b = tb; b < nb; b += PG_NI) {
            const int st = (int)(b % PG_D);
            if (pg_aborted(sh)) break;
            if (!pg_wait(sh, &sh.full[st], (uint32_t)((b / PG_D) & 1), err)) break;
#pragma unroll
            for (int k = 0; k < PG_N / 32; ++k) {        // rows lane, lane + 32: 16 nibble bytes -> 2 chunks of int8 (q - 8)
                const int n = lane + 32 * k;
                const uint4 w = *reinterpret_cast<const uint4 *>(sh.nib[st] + n * 16);
                const uint4 lo = make_uint4(__vsub4(w.x & 0x0F0F0F0Fu, 0x08080808u), __vsub4(w.y & 0x0F0F0F0Fu, 0x08080808u),
                                            __vsub4(w.z & 0x0F0F0F0Fu, 0x08080808u), __vsub4(w.w & 0x0F0F0F0Fu, 0x08080808u));
                const uint4 hi = make_uint4(__vsub4((w.x >> 4) & 0x0F0F0F0Fu, 0x08080808u),
                                            __vsub4((w.y >> 4) & 0x0F0F0F0Fu, 0x08080808u),
                                            __vsub4((w.z >> 4) & 0x0F0F0F0Fu, 0x08080808u),
                                            __vsub4((w.w >> 4) & 0x0F0F0F0Fu, 0x08080808u));
                *reinterpret_cast<uint4 *>(sh.b[st] + pg_off(n, 0)) = lo;
                *reinterpret_cast<uint4 *>(sh.b[st] + pg_off(n, 1)) = hi;
                sh.dwf[st][n] = alb_h2f(sh.dws[(b >> 3) & 1][n][b & 7]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic stores -> tensor core
            __syncwarp();
            if (!pg_wait(sh, &sh.tempty[tb], (uint32_t)((b / PG_NB) & 1), err)) break;   // phase 0: the first bias fill
            if (lane == 0) {
                pg_fence_after();
                const uint64_t da = pg_desc(sh.a[st]), db = pg_desc(sh.b[st]);
                const uint32_t accumulate = 1, zero = 0;   // D = bias + A.B
                asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                             "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
                             :: "r"(tmem + (uint32_t)(tb * PG_N)), "l"(da), "l"(db), "r"(PG_IDESC), "r"(accumulate), "r"(zero)
                             : "memory");
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                             :: "r"(pg_smem(&sh.tfull[tb])) : "memory");
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                             :: "r"(pg_smem(&sh.empty[st])) : "memory");
                alb_mbar_arrive(&sh.tfull[tb]);   // release: this block's dwf (and the loads this warp observed)
            }
            __syncwarp();
        }
        if (lane == 0) {   // every MMA issued by this thread complete (the TMEM is freed below)
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         :: "r"(pg_smem(&sh.drain)) : "memory");
            pg_wait(sh, &sh.drain, 0u, err);
        }
        __syncwarp();
    } else {
        // --------------------------------------------------- epilogue warps
        {   // every buffer's columns of this warp <- the bias; tempty phase 0
            const uint32_t t0 = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(chalf * 32);
            for (int k = 0; k < PG_NB; ++k) {
                pg_tmem_fill16(t0 + (uint32_t)(k * PG_N), PG_BIAS);
                pg_tmem_fill16(t0 + (uint32_t)(k * PG_N + 16), PG_BIAS);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            pg_fence_before();
            __syncwarp();
            if (lane == 0)
                for (int k = 0; k < PG_NB; ++k) alb_mbar_arrive(&sh.tempty[k]);
        }
        for (int64_t b = 0; b < nb; ++b) {
            const int st = (int)(b % PG_D), tb = (int)(b % PG_NB);
            if (pg_aborted(sh)) break;
            if (!pg_wait(sh, &sh.tfull[tb], (uint32_t)((b / PG_NB) & 1), err)) break;
            pg_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(tb * PG_N + chalf * 32);
            const float dxr = sh.dx[st][row];
            const float * dwp = &sh.dwf[st][chalf * 32];
            // two halves of 16 columns (16 accumulator words live at a time).  The
            // accumulator holds bits(1.5 * 2^23) + I: one fp32 subtract gives
            // float(I); dx * dw is exact (11 x 11 bits)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t c[16];
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                             "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                             : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3]), "=r"(c[4]), "=r"(c[5]), "=r"(c[6]),
                               "=r"(c[7]), "=r"(c[8]), "=r"(c[9]), "=r"(c[10]), "=r"(c[11]), "=r"(c[12]), "=r"(c[13]),
                               "=r"(c[14]), "=r"(c[15])
                             : "r"(taddr + (uint32_t)(16 * hf)));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    const float4 w4 = *reinterpret_cast<const float4 *>(dwp + 16 * hf + 4 * j4);
                    const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int j = 16 * hf + 4 * j4 + u;
                        const float t = __fsub_rn(__uint_as_float(c[4 * j4 + u]), 12582912.0f);
                        acc[j] = __fmaf_rn(t, __fmul_rn(dxr, wv[u]), acc[j]);
                    }
                }
            }
            // the accumulator was read: set the bias again, release the buffer
            // (after the chain steps, when the 16 words of a fill are free registers)
            pg_tmem_fill16(taddr, PG_BIAS);
            pg_tmem_fill16(taddr + 16u, PG_BIAS);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            pg_fence_before();
            __syncwarp();
            if (lane == 0) { alb_mbar_arrive(&sh.tempty[tb]); alb_mbar_arrive(&sh.empty[st]); }   // buffer and scales
        }
    }
    pg_fence_before();
    __syncthreads();
    if (warp == 1) {
        pg_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(PG_TMEM_COLS) : "memory");
    }
    if (warp < PG_E0 || pg_aborted(sh)) return;
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
    return q + (size_t)pg_mpad(M) * (K / 32) * 4;
}

// x fp32 [M][K] (already normalized if needed) -> y: workspace prefill_ws_bytes(M, K)
cudaError_t launch_prefill_gemm(const uint8_t * W, int64_t N, int64_t K, const float * x, const void * xq_blocks,
                                int64_t M, float * y, int64_t y_stride, const float * residual, bool swiglu, void * ws,
                                int * err, bool pdl, cudaStream_t st) {
    int8_t * xq = reinterpret_cast<int8_t *>(ws);
    float * xd = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(ws) + (((size_t)M * K + 255) & ~(size_t)255));   // [K/32][pg_mpad(M)]
    const int64_t nblk = M * (K / 32);
    cudaError_t e;
    if (x) e = alb_launch(k_pg_quant, dim3((unsigned)((nblk + 7) / 8)), dim3(256), 0, st, pdl, x, M, K, xq, xd);
    else e = alb_launch(k_pg_from_q8, dim3((unsigned)((nblk + 255) / 256)), dim3(256), 0, st, pdl,
                        reinterpret_cast<const uint8_t *>(xq_blocks), M, K, xq, xd);
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)((N + PG_N - 1) / PG_N), (unsigned)((M + PG_M - 1) / PG_M));
    const uint8_t * Ws = W + K / 2;   // scales of row n at Ws + n * q4_row_bytes(K)
    const size_t smem = sizeof(PgShared);
    if (swiglu) {
        e = ensure_smem(k_prefill_gemm<1>, smem);
        if (e != cudaSuccess) return e;
        return alb_launch(k_prefill_gemm<1>, grid, dim3(PG_THREADS), smem, st, pdl, W, Ws, N, K, (const int8_t *)xq,
                          (const float *)xd, M, y, y_stride, residual, err);
    }
    e = ensure_smem(k_prefill_gemm<0>, smem);
    if (e != cudaSuccess) return e;
    return alb_launch(k_prefill_gemm<0>, grid, dim3(PG_THREADS), smem, st, pdl, W, Ws, N, K, (const int8_t *)xq,
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
