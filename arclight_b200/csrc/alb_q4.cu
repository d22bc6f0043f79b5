// Q4_0 x Q8_0 mat-vec for batch-1 decode, Q8_0 quantization and the Q4_0 GPU
// layout (sm_100a).
//
// Reference semantics: nnml_gemv_q4_0_4x4_q8_0 (nnml/src/ops/arm/gemm.cpp:127-190)
// driven by forward_mul_mat (nnml/src/ops/arm/arm.cpp:1855-1925); activations
// quantized by quantize_row_q8_0 (arm.cpp:1819-1853).
//
// Design: the weight is HBM-bound streamed once.  The GPU layout splits each
// row into a 16-byte-per-block nibble plane and an fp16 scale plane so a warp
// reads 512 contiguous bytes per step with 16-byte non-allocating loads.  One
// warp owns one row (or a gate/up row pair); lanes stride over the K/32 blocks;
// a 32-value block dot is 8 dp4a on the raw nibbles minus 8 * sum(a), which is
// the reference's int32 I(n,b) exactly.  The Q8_0 activation lives in shared
// memory in a padded 48-byte record per block (conflict-free 128-bit reads).
// Weight loads of a warp's first row are issued before griddepcontrol.wait so
// they overlap the previous kernel's tail under programmatic dependent launch.
#include <cstdio>
#include <cstdlib>

#include "alb_q4_dev.cuh"

namespace alb {



// ---------------------------------------------------------------- repack
// block_q4_0 [N][K/32] (18-byte blocks) <-> nibble plane + pitched scale plane.
__global__ void k_repack_q4_0(uint8_t * __restrict__ dst, const uint8_t * __restrict__ src,
                              int64_t n_blocks, int64_t nb, int64_t spitch, size_t scale_off) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_blocks) return;
    const uint16_t * s = reinterpret_cast<const uint16_t *>(src + i * 18);  // 2-byte aligned
    uint16_t q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = s[1 + j];
    uint4 v;
    v.x = (uint32_t)q[0] | ((uint32_t)q[1] << 16);
    v.y = (uint32_t)q[2] | ((uint32_t)q[3] << 16);
    v.z = (uint32_t)q[4] | ((uint32_t)q[5] << 16);
    v.w = (uint32_t)q[6] | ((uint32_t)q[7] << 16);
    reinterpret_cast<uint4 *>(dst)[i] = v;
    const int64_t row = i / nb, b = i - row * nb;
    uint16_t * sc = reinterpret_cast<uint16_t *>(dst + scale_off) + row * spitch;
    sc[b] = s[0];
    if (b == nb - 1)
        for (int64_t j = nb; j < spitch; ++j) sc[j] = 0;   // defined padding
}

__global__ void k_unpack_q4_0(uint8_t * __restrict__ dst, const uint8_t * __restrict__ src,
                              int64_t n_blocks, int64_t nb, int64_t spitch, size_t scale_off) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_blocks) return;
    const uint4 v = reinterpret_cast<const uint4 *>(src)[i];
    uint16_t * d = reinterpret_cast<uint16_t *>(dst + i * 18);
    const int64_t row = i / nb, b = i - row * nb;
    d[0] = reinterpret_cast<const uint16_t *>(src + scale_off)[row * spitch + b];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) { d[1 + 2 * j] = (uint16_t)(w[j] & 0xFFFF); d[2 + 2 * j] = (uint16_t)(w[j] >> 16); }
}

__global__ void k_quantize_q8_0(const float * __restrict__ x, uint8_t * __restrict__ y, int64_t n_blocks) {
    const int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    alb_pdl_wait();
    if (b < n_blocks) {
        int8_t q; uint16_t dh;
        q8_block_lane(x[b * 32 + lane], q, dh);
        uint8_t * blk = y + b * 34;
        if (lane == 0) *reinterpret_cast<uint16_t *>(blk) = dh;
        blk[2 + lane] = (uint8_t)q;
    }
    alb_pdl_trigger();
}

cudaError_t launch_quantize_q8_0(const float * x, void * xq, int64_t n, bool pdl, cudaStream_t st) {
    const int64_t nb = n / 32;
    return alb_launch(k_quantize_q8_0, dim3((unsigned)((nb + 7) / 8)), dim3(256), 0, st, pdl, x,
                      static_cast<uint8_t *>(xq), nb);
}

// CONSUMERS_ONLY: synchronise the GEMV_WARPS consumer warps with named barrier 1
// (the producer warp of the bulk-copy kernel does not take part).
template <int IN, bool CONSUMERS_ONLY>
__device__ __forceinline__ void gemv_prologue_impl(const GemvArgs & a, int * xs, int nb, uint4 * stage) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if constexpr (IN == GEMV_IN_Q8) {
        // stage the block_q8_0 vector (16-byte loads when aligned; never past
        // its nb*34 bytes), then unpack per block
        const int nbytes = nb * 34;
        if ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0) {
            const int n16 = nbytes / 16;
            const uint4 * src = static_cast<const uint4 *>(a.x);
            for (int i = tid; i < n16; i += GEMV_WARPS * 32) stage[i] = src[i];
            for (int i = n16 * 16 + tid; i < nbytes; i += GEMV_WARPS * 32)
                reinterpret_cast<uint8_t *>(stage)[i] = static_cast<const uint8_t *>(a.x)[i];
        } else {
            for (int i = tid; i < nbytes; i += GEMV_WARPS * 32)
                reinterpret_cast<uint8_t *>(stage)[i] = static_cast<const uint8_t *>(a.x)[i];
        }
        if constexpr (CONSUMERS_ONLY) asm volatile("bar.sync 1, %0;" :: "n"(GEMV_WARPS * 32) : "memory");
        else __syncthreads();
        const uint8_t * xq = reinterpret_cast<const uint8_t *>(stage);
        for (int b = tid; b < nb; b += GEMV_WARPS * 32) {
            const uint16_t * s = reinterpret_cast<const uint16_t *>(xq + (size_t)b * 34);
            int * rec = xs + b * XREC_INTS;
            int sum = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t v = (uint32_t)s[1 + 2 * k] | ((uint32_t)s[2 + 2 * k] << 16);
                rec[k] = (int)v;
                sum += (int8_t)(v & 0xFF) + (int8_t)((v >> 8) & 0xFF) + (int8_t)((v >> 16) & 0xFF) + (int8_t)(v >> 24);
            }
            rec[8] = __float_as_int(alb_h2f(s[0]));
            rec[9] = sum;
        }
    } else {
        // x (and the norm weights) staged in shared memory with 16-byte copies,
        // then the sum of squares in a 256-thread strided order and the blocks
        // quantized from shared memory (no dependent global loads per block)
        const float * x = static_cast<const float *>(a.x);
        float * xf = reinterpret_cast<float *>(stage);
        float * wf = xf + a.K;   // RMS only
        const int K = (int)a.K;
        const bool vec = (K & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                         (IN != GEMV_IN_F32_RMS || (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0);
        if (vec) {
            const float4 * x4 = reinterpret_cast<const float4 *>(x);
            const float4 * w4 = reinterpret_cast<const float4 *>(a.norm_w);
            for (int i = tid; i < K / 4; i += GEMV_WARPS * 32) {
                reinterpret_cast<float4 *>(xf)[i] = x4[i];
                if constexpr (IN == GEMV_IN_F32_RMS) reinterpret_cast<float4 *>(wf)[i] = w4[i];
            }
        } else {
            for (int i = tid; i < K; i += GEMV_WARPS * 32) {
                xf[i] = x[i];
                if constexpr (IN == GEMV_IN_F32_RMS) wf[i] = a.norm_w[i];
            }
        }
        if constexpr (CONSUMERS_ONLY) asm volatile("bar.sync 1, %0;" :: "n"(GEMV_WARPS * 32) : "memory");
        else __syncthreads();
        float scale = 1.0f;
        if constexpr (IN == GEMV_IN_F32_RMS) {
            // sum of float squares accumulated in double (ops.cpp:703-710)
            __shared__ double red[GEMV_WARPS];
            double s = 0.0;
            for (int i = tid; i < K; i += GEMV_WARPS * 32) { const float v = xf[i]; s += (double)__fmul_rn(v, v); }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) red[warp] = s;
            if constexpr (CONSUMERS_ONLY) asm volatile("bar.sync 1, %0;" :: "n"(GEMV_WARPS * 32) : "memory");
            else __syncthreads();
            double t = 0.0;
#pragma unroll
            for (int w = 0; w < GEMV_WARPS; ++w) t += red[w];
            const float mean = (float)(t / (double)a.K);
            scale = 1.0f / sqrtf(__fadd_rn(mean, a.eps));
        }
        for (int b = warp; b < nb; b += GEMV_WARPS) {
            float v = xf[b * 32 + lane];
            if constexpr (IN == GEMV_IN_F32_RMS) v = __fmul_rn(__fmul_rn(v, scale), wf[b * 32 + lane]);
            int8_t q; uint16_t dh;
            q8_block_lane(v, q, dh);
            store_xrec(xs, b, lane, q, dh);
        }
    }
}

// Shared memory after the activation records: the raw block_q8_0 vector
// (IN_Q8) or the fp32 input (and norm weights) of the prologue.
__host__ __device__ inline size_t gemv_stage_bytes(int64_t K, int in_mode) {
    const size_t q8 = ((size_t)(K / 32) * 34 + 15) / 16 * 16;
    const size_t f32 = in_mode == GEMV_IN_F32 ? (size_t)K * 4 : in_mode == GEMV_IN_F32_RMS ? (size_t)K * 8 : 0;
    return q8 > f32 ? q8 : f32;
}

template <int IN>
__device__ __forceinline__ void gemv_prologue(const GemvArgs & a, int * xs, int nb, uint4 * stage) {
    gemv_prologue_impl<IN, false>(a, xs, nb, stage);
}
template <int IN>
__device__ __forceinline__ void gemv_prologue_bar(const GemvArgs & a, int * xs, int nb, uint4 * stage) {
    gemv_prologue_impl<IN, true>(a, xs, nb, stage);
}

// L2 prefetch of [p, p + bytes) in <= 64 KiB bulk requests (16-byte granules).
__device__ __forceinline__ void l2_prefetch(const void * p, size_t bytes) {
    const uint8_t * c = static_cast<const uint8_t *>(p);
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(c) & ~(uintptr_t)15;
    const uintptr_t a1 = (reinterpret_cast<uintptr_t>(c) + bytes + 15) & ~(uintptr_t)15;
    for (uintptr_t a = a0; a < a1; a += 65536) {
        const uint32_t n = (uint32_t)((a1 - a) < 65536 ? (a1 - a) : 65536);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(a), "r"(n) : "memory");
    }
}

// After lane 0 wrote the SwiGLU output y[item]: with a.yq set, the warp whose
// value completes a 32-value block quantizes that block (quantize_row_q8_0 of
// the fp32 values, the down projection's input) and re-arms its counter.
// Writers publish y before their arrival (fence + atomic); the last one reads
// the block from L2 after its own fence.  Called by the whole warp.
__device__ __forceinline__ void gemv_swiglu_q8_tail(const GemvArgs & a, int64_t item, int lane) {
    if (!a.yq) return;
    const int64_t b = item >> 5;
    int last = 0;
    if (lane == 0) {
        __threadfence();
        last = atomicAdd(&a.ycnt[b], 1) == 31;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    const float v = __ldcg(a.y + b * 32 + lane);
    int8_t q; uint16_t dh;
    q8_block_lane(v, q, dh);
    uint8_t * blk = a.yq + b * 34;
    if (lane == 0) {
        *reinterpret_cast<uint16_t *>(blk) = dh;
        a.ycnt[b] = 0;
    }
    blk[2 + lane] = (uint8_t)q;
}

// Each CTA owns a contiguous range of row items; before waiting on the previous
// kernel it asks the TMA unit to pull its whole weight range (nibbles and
// scales, in PF-byte windows ahead of the compute) into L2, and each warp loads
// its first item into registers.  The compute loop then mostly hits L2.
template <int ITERS, int RPW, int IN, int OUT>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
k_gemv_direct(const GemvArgs a) {
    extern __shared__ int4 smem_i4[];
    int * xs = reinterpret_cast<int *>(smem_i4);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = (int)(a.K / 32);
    const size_t row_bytes = (size_t)a.K / 2;
    const uint8_t * Wn = a.W;
    const uint16_t * Ws = reinterpret_cast<const uint16_t *>(a.S);
    const int64_t sp = q4_scale_pitch(a.K);
    const int64_t n_items = a.N / RPW;
    const int64_t it0 = n_items * blockIdx.x / gridDim.x;
    const int64_t it1 = n_items * (blockIdx.x + 1) / gridDim.x;
    constexpr size_t PF = 96 * 1024;      // prefetch window per CTA (nibble bytes)
    const size_t item_bytes = row_bytes * RPW;
    int64_t pf_item = it0;                // first item not yet prefetched
    auto prefetch_upto = [&](int64_t item_end) {
        if (item_end > it1) item_end = it1;
        if (item_end <= pf_item) return;
        l2_prefetch(Wn + pf_item * item_bytes, (size_t)(item_end - pf_item) * item_bytes);
        l2_prefetch(Ws + pf_item * RPW * sp, (size_t)(item_end - pf_item) * RPW * sp * 2);
        pf_item = item_end;
    };
    const int64_t pf_items = (int64_t)(PF / item_bytes) + 1;
    if (threadIdx.x == 0) prefetch_upto(it0 + pf_items);

    uint4 w[RPW][ITERS];
    uint16_t dw[RPW][ITERS];
    auto load = [&](int64_t it) {
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const int64_t row = it * RPW + r;
            const uint8_t * wr = Wn + row * row_bytes;
            const uint16_t * sr = Ws + row * sp;
#pragma unroll
            for (int i = 0; i < ITERS; ++i) {
                const int b = lane + 32 * i;
                if (b < nb) { w[r][i] = alb_ld_stream(wr + 16 * b); dw[r][i] = __ldg(sr + b); }
            }
        }
    };
    int64_t item = it0 + warp;
    if (item < it1) load(item);   // weights do not depend on the previous kernel

    alb_pdl_wait();
    gemv_prologue<IN>(a, xs, nb, reinterpret_cast<uint4 *>(xs + nb * XREC_INTS));
    __syncthreads();
    alb_pdl_trigger();

    for (; item < it1; item += GEMV_WARPS) {
        if (warp == 0 && lane == 0) prefetch_upto(item + pf_items);
        double acc[RPW];
#pragma unroll
        for (int r = 0; r < RPW; ++r) acc[r] = 0.0;
#pragma unroll
        for (int i = 0; i < ITERS; ++i) {
            const int b = lane + 32 * i;
            if (b < nb) {
                const int4 * rec = reinterpret_cast<const int4 *>(xs + b * XREC_INTS);
                const int4 a_lo = rec[0], a_hi = rec[1];
                const int2 ds = reinterpret_cast<const int2 *>(rec + 2)[0];
                const float dx = __int_as_float(ds.x);
#pragma unroll
                for (int r = 0; r < RPW; ++r) {
                    const int I = q4q8_dot(w[r][i], a_lo, a_hi, ds.y);
                    if constexpr (OUT == GEMV_OUT_DOTS) a.dots[(item * RPW + r) * nb + b] = I;
                    acc[r] = fma((double)I, (double)__fmul_rn(dx, alb_h2f(dw[r][i])), acc[r]);
                }
            }
        }
        const int64_t cur = item;
        if (item + GEMV_WARPS < it1) load(item + GEMV_WARPS);  // next item's weights in flight
#pragma unroll
        for (int r = 0; r < RPW; ++r) acc[r] = alb_warp_sum_d(acc[r]);
        if (lane == 0 && a.y) {
            if constexpr (OUT == GEMV_OUT_SWIGLU) {
                const float g = __double2float_rn(acc[0]), u = __double2float_rn(acc[1]);
                a.y[cur] = alb_swiglu1(g, u);
            } else {
#pragma unroll
                for (int r = 0; r < RPW; ++r) {
                    const int64_t row = cur * RPW + r;
                    const float yv = __double2float_rn(acc[r]);
                    a.y[row] = a.residual ? __fadd_rn(yv, a.residual[row]) : yv;
                }
            }
        }
        if constexpr (OUT == GEMV_OUT_SWIGLU) gemv_swiglu_q8_tail(a, cur, lane);
    }
}

// ---------------------------------------------------------------- bulk-copy pipeline
// One producer warp streams the CTA's contiguous row range through an NS-stage
// shared-memory ring with cp.async.bulk (16-byte aligned 1-D copies, one for
// the nibbles and one for the scales of GEMV_WARPS*RPW rows, completion counted
// on the stage's mbarrier).  It never waits on the previous kernel: under PDL
// the first NS stages are in flight while the previous grid drains.  The
// GEMV_WARPS consumer warps wait (bounded) on the full barrier, each computes
// its RPW rows of the stage from shared memory and releases the slot.
struct TmaPlan {
    int ns;            // stages
    int rs;            // rows per stage
    uint32_t nib_bytes, sc_bytes, stage_bytes, xs_bytes;
    size_t smem;
};

__host__ __device__ inline TmaPlan tma_plan(int64_t K, int rpw, int max_stage_budget, int in_mode) {
    TmaPlan p;
    const int64_t nb = K / 32;
    p.rs = GEMV_WARPS * rpw;
    p.nib_bytes = (uint32_t)(p.rs * (K / 2));
    p.sc_bytes = (uint32_t)(p.rs * q4_scale_pitch(K) * 2);
    p.stage_bytes = p.nib_bytes + p.sc_bytes;
    p.ns = (int)(max_stage_budget / p.stage_bytes);
    if (p.ns < 2) p.ns = 2;
    if (p.ns > 8) p.ns = 8;
    p.xs_bytes = (uint32_t)(nb * XREC_INTS * 4 + gemv_stage_bytes(K, in_mode));
    p.smem = (size_t)p.ns * p.stage_bytes + p.xs_bytes + 2 * 8 * p.ns;
    return p;
}

template <int ITERS, int RPW, int IN, int OUT>
__global__ void __launch_bounds__((GEMV_WARPS + 1) * 32)
k_gemv_tma(const GemvArgs a, const TmaPlan plan) {
    extern __shared__ int4 smem_i4[];
    uint8_t * smem = reinterpret_cast<uint8_t *>(smem_i4);
    uint8_t * stages = smem;
    int * xs = reinterpret_cast<int *>(smem + (size_t)plan.ns * plan.stage_bytes);
    uint64_t * full = reinterpret_cast<uint64_t *>(smem + (size_t)plan.ns * plan.stage_bytes + plan.xs_bytes);
    uint64_t * empty = full + plan.ns;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = (int)(a.K / 32);
    const int64_t sp = q4_scale_pitch(a.K);
    const size_t row_bytes = (size_t)a.K / 2;
    const int64_t n_items = a.N / RPW;
    const int64_t it0 = n_items * blockIdx.x / gridDim.x;
    const int64_t it1 = n_items * (blockIdx.x + 1) / gridDim.x;
    const int n_groups = (int)((it1 - it0 + GEMV_WARPS - 1) / GEMV_WARPS);
    const int NS = plan.ns;

    if (threadIdx.x == GEMV_WARPS * 32) {
        for (int i = 0; i < NS; ++i) { alb_mbar_init(&full[i], 1); alb_mbar_init(&empty[i], GEMV_WARPS); }
        alb_mbar_fence_init();
    }
    __syncthreads();

    if (warp == GEMV_WARPS) {
        // ------------------------------------------------ producer warp
        if (lane == 0) {
            bool ok = true;
            int issued = 0;
            for (int g = 0; g < n_groups && ok; ++g) {
                const int st = g % NS;
                if (g >= NS && !alb_mbar_wait(&empty[st], (uint32_t)((g / NS - 1) & 1))) { ok = false; break; }
                const int64_t ig = it0 + (int64_t)g * GEMV_WARPS;
                const int64_t items = (it1 - ig) < GEMV_WARPS ? (it1 - ig) : GEMV_WARPS;
                const int64_t r0 = ig * RPW, rows = items * RPW;
                const uint32_t nbytes = (uint32_t)(rows * row_bytes), sbytes = (uint32_t)(rows * sp * 2);
                uint8_t * dst = stages + (size_t)st * plan.stage_bytes;
                alb_mbar_expect_tx(&full[st], nbytes + sbytes);
                alb_bulk_g2s(dst, a.W + r0 * row_bytes, nbytes, &full[st]);
                alb_bulk_g2s(dst + plan.nib_bytes, a.S + r0 * sp * 2, sbytes, &full[st]);
                issued = g + 1;
            }
            if (!ok) atomicExch(a.err, ALB_DEVERR_MBAR_TIMEOUT);
            // never leave with copies in flight: the last stages' phases must complete
            for (int g = issued - NS < 0 ? 0 : issued - NS; g < issued; ++g)
                alb_mbar_wait(&full[g % NS], (uint32_t)((g / NS) & 1));
        }
        return;
    }

    // ---------------------------------------------------- consumer warps
    alb_pdl_wait();
    gemv_prologue_bar<IN>(a, xs, nb, reinterpret_cast<uint4 *>(xs + nb * XREC_INTS));
    asm volatile("bar.sync 1, %0;" :: "n"(GEMV_WARPS * 32) : "memory");
    alb_pdl_trigger();

    for (int g = 0; g < n_groups; ++g) {
        const int st = g % NS;
        if (!alb_mbar_wait(&full[st], (uint32_t)((g / NS) & 1))) {
            if (lane == 0) atomicExch(a.err, ALB_DEVERR_MBAR_TIMEOUT);
            break;
        }
        const int64_t item = it0 + (int64_t)g * GEMV_WARPS + warp;
        if (item < it1) {
            const uint8_t * nib = stages + (size_t)st * plan.stage_bytes + (size_t)warp * RPW * row_bytes;
            const uint16_t * sc = reinterpret_cast<const uint16_t *>(stages + (size_t)st * plan.stage_bytes + plan.nib_bytes) + (size_t)warp * RPW * sp;
            double acc[RPW];
#pragma unroll
            for (int r = 0; r < RPW; ++r) acc[r] = 0.0;
#pragma unroll
            for (int i = 0; i < ITERS; ++i) {
                const int b = lane + 32 * i;
                if (b < nb) {
                    const int4 * rec = reinterpret_cast<const int4 *>(xs + b * XREC_INTS);
                    const int4 a_lo = rec[0], a_hi = rec[1];
                    const int2 ds = reinterpret_cast<const int2 *>(rec + 2)[0];
                    const float dx = __int_as_float(ds.x);
#pragma unroll
                    for (int r = 0; r < RPW; ++r) {
                        const uint4 w = *reinterpret_cast<const uint4 *>(nib + r * row_bytes + 16 * b);
                        const int I = q4q8_dot(w, a_lo, a_hi, ds.y);
                        acc[r] = fma((double)I, (double)__fmul_rn(dx, alb_h2f(sc[r * sp + b])), acc[r]);
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < RPW; ++r) acc[r] = alb_warp_sum_d(acc[r]);
            if (lane == 0) {
                if constexpr (OUT == GEMV_OUT_SWIGLU) {
                    const float gt = __double2float_rn(acc[0]), u = __double2float_rn(acc[1]);
                    a.y[item] = alb_swiglu1(gt, u);
                } else {
#pragma unroll
                    for (int r = 0; r < RPW; ++r) {
                        const int64_t row = item * RPW + r;
                        const float yv = __double2float_rn(acc[r]);
                    a.y[row] = a.residual ? __fadd_rn(yv, a.residual[row]) : yv;
                    }
                }
            }
            if constexpr (OUT == GEMV_OUT_SWIGLU) gemv_swiglu_q8_tail(a, item, lane);
        }
        __syncwarp();
        if (lane == 0) alb_mbar_arrive(&empty[st]);
    }
}

template <int ITERS, int RPW, int IN, int OUT>
static cudaError_t launch_gemv_t(const GemvArgs & a, cudaStream_t stream) {
    const int nb = (int)(a.K / 32);
    const int64_t items = a.N / RPW;
    const bool direct = (OUT == GEMV_OUT_DOTS) || a.variant != 2;
    if (direct) {
        auto kern = k_gemv_direct<ITERS, RPW, IN, OUT>;
        const size_t smem = (size_t)nb * XREC_INTS * 4 + gemv_stage_bytes(a.K, IN);
        static size_t attr_smem = 0;   // per instantiation
        if (smem > 48 * 1024 && smem > attr_smem) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            attr_smem = smem;
        }
        const int per_sm = a.ctas_per_sm > 0 ? a.ctas_per_sm : 3;
        int64_t grid = (int64_t)alb_sm_count() * per_sm;
        if (grid * GEMV_WARPS > items) grid = (items + GEMV_WARPS - 1) / GEMV_WARPS;
        if (grid < 1) grid = 1;
        return alb_launch(kern, dim3((unsigned)grid), dim3(GEMV_WARPS * 32), smem, stream, a.pdl, a);
    }
    auto kern = k_gemv_tma<ITERS, RPW, IN, OUT>;
    const TmaPlan plan = tma_plan(a.K, RPW, a.stage_budget > 0 ? a.stage_budget : 88 * 1024, IN);
    static size_t attr_smem = 0;
    if (plan.smem > attr_smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem);
        if (e != cudaSuccess) return e;
        attr_smem = plan.smem;
    }
    const int per_sm = a.ctas_per_sm > 0 ? a.ctas_per_sm : 1;
    int64_t grid = (int64_t)alb_sm_count() * per_sm;
    if (grid * GEMV_WARPS > items) grid = (items + GEMV_WARPS - 1) / GEMV_WARPS;
    if (grid < 1) grid = 1;
    return alb_launch(kern, dim3((unsigned)grid), dim3((GEMV_WARPS + 1) * 32), plan.smem, stream, a.pdl, a, plan);
}

template <int ITERS, int IN, int OUT>
static cudaError_t dispatch_rpw(const GemvArgs & a, cudaStream_t s) {
    constexpr int RPW = (OUT == GEMV_OUT_SWIGLU) ? 2 : (ITERS <= 5 ? 2 : 1);
    if (a.N % RPW != 0) return launch_gemv_t<ITERS, 1, IN, OUT == GEMV_OUT_SWIGLU ? GEMV_OUT_PLAIN : OUT>(a, s);
    return launch_gemv_t<ITERS, RPW, IN, OUT>(a, s);
}

template <int IN, int OUT>
static cudaError_t dispatch_iters(const GemvArgs & a, cudaStream_t s) {
    const int it = (int)((a.K / 32 + 31) / 32);
    switch (it) {
        case 1: return dispatch_rpw<1, IN, OUT>(a, s);
        case 2: return dispatch_rpw<2, IN, OUT>(a, s);
        case 3: return dispatch_rpw<3, IN, OUT>(a, s);
        case 4: return dispatch_rpw<4, IN, OUT>(a, s);
        case 5: return dispatch_rpw<5, IN, OUT>(a, s);
        case 6: return dispatch_rpw<6, IN, OUT>(a, s);
        case 7: case 8: return dispatch_rpw<8, IN, OUT>(a, s);
        case 9: case 10: return dispatch_rpw<10, IN, OUT>(a, s);
        case 11: case 12: return dispatch_rpw<12, IN, OUT>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(const GemvArgs & a_in, cudaStream_t s) {
    GemvArgs a = a_in;
    if (!a.err) a.err = device_error_ptr();
    if (!a.err) return cudaErrorMemoryAllocation;
    if (a.K % 32 != 0 || a.K <= 0 || a.N <= 0 || a.K > 12288) return cudaErrorInvalidValue;
    if (a.out_mode == GEMV_OUT_SWIGLU && a.N % 2 != 0) return cudaErrorInvalidValue;
    if (a.yq && (a.out_mode != GEMV_OUT_SWIGLU || !a.ycnt || !a.y || (a.N / 2) % 32 != 0)) return cudaErrorInvalidValue;
#define ALB_GEMV_CASE(IN)                                                           \
    case IN:                                                                        \
        switch (a.out_mode) {                                                       \
            case GEMV_OUT_PLAIN: return dispatch_iters<IN, GEMV_OUT_PLAIN>(a, s);   \
            case GEMV_OUT_SWIGLU: return dispatch_iters<IN, GEMV_OUT_SWIGLU>(a, s); \
            case GEMV_OUT_DOTS: return dispatch_iters<IN, GEMV_OUT_DOTS>(a, s);     \
            default: return cudaErrorInvalidValue;                                  \
        }
    switch (a.in_mode) {
        ALB_GEMV_CASE(GEMV_IN_Q8)
        ALB_GEMV_CASE(GEMV_IN_F32)
        ALB_GEMV_CASE(GEMV_IN_F32_RMS)
        default: return cudaErrorInvalidValue;
    }
#undef ALB_GEMV_CASE
}

}  // namespace alb

// ================================================================ C ABI
using namespace alb;

// Tuning knobs for the standalone C-ABI mat-vec (read once per process):
//   ALB_GEMV_VARIANT=1|2 (direct loads + L2 prefetch | bulk-copy pipeline),
//   ALB_GEMV_CTAS=<CTAs per SM>, ALB_GEMV_STAGE_KB=<shared-memory stage budget>,
//   ALB_GEMV_PDL=0|1 (programmatic dependent launch, default 1).
static void apply_gemv_knobs(GemvArgs & a) {
    static int variant = -1, ctas = 0, stage_kb = 0, pdl = 1;
    if (variant < 0) {
        const char * p = getenv("ALB_GEMV_PDL");
        pdl = p ? atoi(p) : 1;
        const char * v = getenv("ALB_GEMV_VARIANT");
        const char * c = getenv("ALB_GEMV_CTAS");
        const char * k = getenv("ALB_GEMV_STAGE_KB");
        variant = v ? atoi(v) : 1;
        ctas = c ? atoi(c) : 0;
        stage_kb = k ? atoi(k) : 0;
    }
    a.variant = variant;
    a.ctas_per_sm = ctas;
    a.stage_budget = stage_kb * 1024;
    a.pdl = pdl != 0;
}

extern "C" size_t alb_q4_0_gpu_bytes(int64_t N, int64_t K) { return q4_gpu_bytes(N, K); }
extern "C" size_t alb_q4_0_scale_offset(int64_t N, int64_t K) { return q4_scale_offset(N, K); }

extern "C" int alb_repack_q4_0(void * dst, const void * src, int64_t N, int64_t K, void * stream) {
    ALB_CHECK_ARG(dst && src && N > 0 && K > 0 && K % 32 == 0);
    const int64_t nbk = N * (K / 32);
    k_repack_q4_0<<<(unsigned)((nbk + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (uint8_t *)dst, (const uint8_t *)src, nbk, K / 32, q4_scale_pitch(K), q4_scale_offset(N, K));
    ALB_CUDA_TRY(cudaGetLastError());
    return ALB_OK;
}

extern "C" int alb_unpack_q4_0(void * dst, const void * src, int64_t N, int64_t K, void * stream) {
    ALB_CHECK_ARG(dst && src && N > 0 && K > 0 && K % 32 == 0);
    const int64_t nbk = N * (K / 32);
    k_unpack_q4_0<<<(unsigned)((nbk + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (uint8_t *)dst, (const uint8_t *)src, nbk, K / 32, q4_scale_pitch(K), q4_scale_offset(N, K));
    ALB_CUDA_TRY(cudaGetLastError());
    return ALB_OK;
}

extern "C" int alb_quantize_q8_0(const float * x, void * xq, int64_t K, int64_t rows, void * stream) {
    ALB_CHECK_ARG(x && xq && K > 0 && K % 32 == 0 && rows > 0);
    const int64_t nbk = rows * (K / 32);
    k_quantize_q8_0<<<(unsigned)((nbk * 32 + 255) / 256), 256, 0, (cudaStream_t)stream>>>(x, (uint8_t *)xq, nbk);
    ALB_CUDA_TRY(cudaGetLastError());
    return ALB_OK;
}

extern "C" int alb_gemv_q4_0_q8_0(const void * W, const void * xq, float * y, int64_t N, int64_t K,
                                  const float * residual, void * stream) {
    ALB_CHECK_ARG(W && xq && y && N > 0 && K > 0 && K % 32 == 0 && K <= 12288);
    GemvArgs a;
    a.W = (const uint8_t *)W; a.S = (const uint8_t *)W + q4_scale_offset(N, K); a.N = N; a.K = K;
    a.in_mode = GEMV_IN_Q8; a.x = xq;
    a.out_mode = GEMV_OUT_PLAIN; a.y = y; a.residual = residual;
    a.pdl = true;
    apply_gemv_knobs(a);
    ALB_CUDA_TRY(launch_gemv(a, (cudaStream_t)stream));
    return ALB_OK;
}

extern "C" int alb_gemv_q4_0_q8_0_block_dots(const void * W, const void * xq, int32_t * I, int64_t N, int64_t K,
                                             void * stream) {
    ALB_CHECK_ARG(W && xq && I && N > 0 && K > 0 && K % 32 == 0 && K <= 12288);
    GemvArgs a;
    a.W = (const uint8_t *)W; a.S = (const uint8_t *)W + q4_scale_offset(N, K); a.N = N; a.K = K;
    a.in_mode = GEMV_IN_Q8; a.x = xq;
    a.out_mode = GEMV_OUT_DOTS; a.dots = I; a.y = nullptr;
    ALB_CUDA_TRY(launch_gemv(a, (cudaStream_t)stream));
    return ALB_OK;
}
