// Q4_0 x Q8_0 mat-vec for batch-1 decode, Q8_0 quantization and the Q4_0 GPU
// layout (sm_100a).
//
// Reference semantics: nnml_gemv_q4_0_4x4_q8_0 (nnml/src/ops/arm/gemm.cpp:127-190)
// driven by forward_mul_mat (arm.cpp:1855-1925) for the projections, and
// nnml_vec_dot_q4_0_q8_0 (arm.cpp:401-692) driven by forward_mul_mat_generic
// (common.cpp:120-248) for the lm head; activations quantized by
// quantize_row_q8_0 (arm.cpp:1819-1853).  The GPU computes the same fp32 fma
// chains in the same block order, so every output is bit-identical to the
// reference's NEON arithmetic (the int32 block dots are exact integers either
// way; only the order of the fp32 accumulation matters).
//
// Design: the weights are HBM-bound and streamed once, by bulk copies into a
// shared-memory ring issued before the kernel waits on its predecessor; the
// block dots are computed in parallel from shared memory (8 dp4a per block on
// the raw nibbles minus 8 * sum(a)), and the short fp32 chains run one lane per
// row over the staged exact terms.
#include <cstdio>
#include <cstdlib>

#include "alb_q4_dev.cuh"

namespace alb {



// ---------------------------------------------------------------- repack
// block_q4_0 [N][K/32] (18-byte blocks) <-> the row-interleaved GPU layout.
__global__ void k_repack_q4_0(uint8_t * __restrict__ dst, const uint8_t * __restrict__ src,
                              int64_t n_blocks, int64_t nb, int64_t spitch, int64_t rowb) {
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
    const int64_t row = i / nb, b = i - row * nb;
    *reinterpret_cast<uint4 *>(dst + row * rowb + 16 * b) = v;
    uint16_t * sc = reinterpret_cast<uint16_t *>(dst + row * rowb + nb * 16);
    sc[b] = s[0];
    if (b == nb - 1)
        for (int64_t j = nb; j < spitch; ++j) sc[j] = 0;   // defined padding
}

__global__ void k_unpack_q4_0(uint8_t * __restrict__ dst, const uint8_t * __restrict__ src,
                              int64_t n_blocks, int64_t nb, int64_t rowb) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_blocks) return;
    const int64_t row = i / nb, b = i - row * nb;
    const uint4 v = *reinterpret_cast<const uint4 *>(src + row * rowb + 16 * b);
    uint16_t * d = reinterpret_cast<uint16_t *>(dst + i * 18);
    d[0] = reinterpret_cast<const uint16_t *>(src + row * rowb + nb * 16)[b];
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

// ---------------------------------------------------------------- mat-vec
// Shared-memory plan of one k_mv launch (computed on the host per K and mode).
//   [0, ns * stage_bytes)        weight stages: R consecutive rows of the GPU
//                                layout [R][q4_row_bytes(K)] (one bulk copy each)
//   cb_off                       chain buffers (ncb of cb_bytes); the prologue's
//                                staging of the input vector aliases them
//   xs_off                       Q8_0 activation records, one per block
//   bar_off                      mbarriers full[ns] empty[ns] done[ncb] free[ncb]
struct MvPlan {
    int R;                  // rows per stage (<= 64; <= 16 for the pair chain)
    int RC;                 // rows per chain-warp pass (32, or 8 for the pair chain)
    int ns, ncb;            // weight stages, chain buffers (ncb == MV_CH: one per chain warp)
    uint32_t stage_bytes;   // R * row bytes
    uint32_t cbp;           // chain-buffer row pitch in bytes (an odd multiple of 16)
    uint32_t cbs;           // pair chain: row pitch of the dx*dw array (an odd number of words)
    uint32_t cb_bytes;      // one chain buffer
    uint32_t cb_off, xs_off, bar_off;
    uint32_t smem;
};

static constexpr int MV_CW = 12;                       // block-dot warps
static constexpr int MV_RU = 3;                        // rows per dot iteration (independent work)
static constexpr int MV_CH = 2;                        // chain warps: stage g goes to chain warp g % MV_CH
static constexpr int MV_PW = MV_CW + MV_CH;            // the producer warp's index
static constexpr int MV_THREADS = (MV_CW + MV_CH + 1) * 32;
static constexpr int MV_NT = (MV_CW + MV_CH) * 32;     // threads of the prologue barrier

// Activation records of the mat-vec: q as 8 packed words, the block scale d
// (fp16-rounded, as float), sum(q), and for the pair chain the four partial
// sums s_l over elements {4l..4l+3} u {16+4l..16+4l+3} (one per vdotq lane).
// Strides of 48 B / 80 B keep the 16-byte reads of 8 consecutive blocks in
// distinct bank groups.
template <bool PAIR> struct XRec { static constexpr int INTS = PAIR ? 20 : 12; };

// quantize_row_q8_0 of one 32-value block by four consecutive threads (the
// block's group of 4 lanes), thread t holding elements 8t..8t+7: amax over the
// block, d = amax / 127, id = 1 / d (0 when d = 0), q = RNE(x * id), d stored
// as fp16 (arm.cpp:1834-1851); writes the mat-vec record (words, d, sum, and
// for the pair chain the four partial sums over {4l..4l+3} u {16+4l..16+4l+3}).
template <bool PAIR>
__device__ __forceinline__ void mv_quant_rec(int * rec, const float (&v)[8], int t, bool on) {
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    int q[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) q[k] = __float2int_rn(__fmul_rn(v[k], id));
    const int w0 = (q[0] & 0xFF) | ((q[1] & 0xFF) << 8) | ((q[2] & 0xFF) << 16) | ((q[3] & 0xFF) << 24);
    const int w1 = (q[4] & 0xFF) | ((q[5] & 0xFF) << 8) | ((q[6] & 0xFF) << 16) | ((q[7] & 0xFF) << 24);
    const int s0 = q[0] + q[1] + q[2] + q[3], s1 = q[4] + q[5] + q[6] + q[7];
    if (on) *reinterpret_cast<int2 *>(rec + 2 * t) = make_int2(w0, w1);
    int s = s0 + s1;
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (on && t == 0) {
        rec[8] = __float_as_int(alb_h2f(alb_f2h(d)));
        rec[9] = s;
    }
    if constexpr (PAIR) {
        // word w of the block is thread w/2's; partial l = word l + word 4 + l
        const int o0 = __shfl_xor_sync(0xffffffffu, s0, 2), o1 = __shfl_xor_sync(0xffffffffu, s1, 2);
        if (on && t < 2) *reinterpret_cast<int2 *>(rec + 10 + 2 * t) = make_int2(s0 + o0, s1 + o1);
    }
}

// dst[0..n) = src[0..n) (16-byte words), by the consumer warps: every load of
// a thread is issued before its stores (one round trip for up to 8 words a
// thread).
__device__ __forceinline__ void mv_stage16(uint4 * dst, const uint4 * __restrict__ src, int n) {
    constexpr int U = 8;
    for (int i0 = 0; i0 < n; i0 += U * MV_NT) {
        uint4 v[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = i0 + threadIdx.x + k * MV_NT;
            if (i < n) v[k] = src[i];
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const int i = i0 + threadIdx.x + k * MV_NT;
            if (i < n) dst[i] = v[k];
        }
    }
}

// Prologue of the consumer warps: the CTA's Q8_0 records of the input vector.
//   IN_Q8     block_q8_0 records from global memory (staged with 16-byte loads);
//   IN_F32    fp32 x quantized here (quantize_row_q8_0, arm.cpp:1819-1853);
//   IN_F32_RMS RMSNorm * w first (ops.cpp:680-724: double sum of the fp32
//             squares, mean rounded to float, 1/sqrtf(mean + eps)); w is
//             already staged at stage + K floats.
// `stage` is scratch of gemv_stage_bytes(K, IN); ends with the consumers'
// named barrier (the producer warp does not take part).
template <int IN, bool PAIR>
__device__ __forceinline__ void mv_prologue(const GemvArgs & a, int * xs, int nb, uint4 * stage) {
    constexpr int XR = XRec<PAIR>::INTS;
    constexpr int NT = MV_NT;
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if constexpr (IN == GEMV_IN_Q8) {
        const int nbytes = nb * 34;
        const uint8_t * src8 = static_cast<const uint8_t *>(a.x);
        if ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0) {
            const int n16 = nbytes / 16;
            const uint4 * src = static_cast<const uint4 *>(a.x);
            mv_stage16(stage, src, n16);
            for (int i = n16 * 16 + tid; i < nbytes; i += NT) reinterpret_cast<uint8_t *>(stage)[i] = src8[i];
        } else {
            for (int i = tid; i < nbytes; i += NT) reinterpret_cast<uint8_t *>(stage)[i] = src8[i];
        }
        asm volatile("bar.sync 1, %0;" :: "n"(NT) : "memory");
        const uint8_t * xq = reinterpret_cast<const uint8_t *>(stage);
        for (int b = tid; b < nb; b += NT) {
            const uint16_t * s = reinterpret_cast<const uint16_t *>(xq + (size_t)b * 34);
            int * rec = xs + b * XR;
            int sum = 0, part[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const uint32_t v = (uint32_t)s[1 + 2 * k] | ((uint32_t)s[2 + 2 * k] << 16);
                rec[k] = (int)v;
                part[k] = (int8_t)(v & 0xFF) + (int8_t)((v >> 8) & 0xFF) + (int8_t)((v >> 16) & 0xFF) + (int8_t)(v >> 24);
                sum += part[k];
            }
            rec[8] = __float_as_int(alb_h2f(s[0]));
            rec[9] = sum;
            if constexpr (PAIR) {
#pragma unroll
                for (int l = 0; l < 4; ++l) rec[10 + l] = part[l] + part[4 + l];
            }
        }
    } else {
        const float * x = static_cast<const float *>(a.x);
        const double inv_k = 1.0 / (double)a.K;   // independent of the loads below
        float * xf = reinterpret_cast<float *>(stage);
        float * wf = xf + a.K;   // the norm weights: staged before the dependency wait
        const int K = (int)a.K;
        if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
            mv_stage16(stage, reinterpret_cast<const uint4 *>(x), K / 4);
        } else {
            for (int i = tid; i < K; i += NT) xf[i] = x[i];
        }
        asm volatile("bar.sync 1, %0;" :: "n"(NT) : "memory");
        float scale = 1.0f;
        if constexpr (IN == GEMV_IN_F32_RMS) {
            // a parallel double sum of the fp32 squares; the reference's
            // sequential sum (ops.cpp:703-710) only where the float mean could differ
            __shared__ double red[NW];
            __shared__ double seq_sum;
            double s = 0.0;
            for (int i = tid; i < K; i += NT) { const float v = xf[i]; s += (double)__fmul_rn(v, v); }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) red[warp] = s;
            asm volatile("bar.sync 1, %0;" :: "n"(NT) : "memory");
            const double t = alb_tree_sum<NW>(red);
            float mean;
            if (!alb_rms_mean_cert(t, K, inv_k, mean)) {   // uniform across the CTA
                if (tid == 0) seq_sum = alb_rms_seq_sum(xf, K);
                asm volatile("bar.sync 1, %0;" :: "n"(NT) : "memory");
                mean = (float)(seq_sum / (double)a.K);
            }
            scale = 1.0f / sqrtf(__fadd_rn(mean, a.eps));
        }
        // quantize_row_q8_0: four threads per block, eight values each (whole
        // warps iterate: the block's four lanes exchange their maxima and sums)
        for (int i0 = warp * 32; i0 < nb * 4; i0 += NT) {
            const int i = i0 + lane, b = i >> 2, t = i & 3;
            const bool on = i < nb * 4;
            float v[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
            if (on) {
                const float4 * x4 = reinterpret_cast<const float4 *>(xf + b * 32 + 8 * t);
                const float4 u0 = x4[0], u1 = x4[1];
                v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w; v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
                if constexpr (IN == GEMV_IN_F32_RMS) {
                    const float4 * w4 = reinterpret_cast<const float4 *>(wf + b * 32 + 8 * t);
                    const float4 z0 = w4[0], z1 = w4[1];
                    const float wv[8] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
#pragma unroll
                    for (int k = 0; k < 8; ++k) v[k] = __fmul_rn(__fmul_rn(v[k], scale), wv[k]);
                }
            }
            mv_quant_rec<PAIR>(xs + b * XR, v, t, on);
        }
    }
    asm volatile("bar.sync 1, %0;" :: "n"(NT) : "memory");
}

// Shared memory of the prologue's staging: the raw block_q8_0 vector (IN_Q8)
// or the fp32 input (and norm weights).
__host__ __device__ inline size_t gemv_stage_bytes(int64_t K, int in_mode) {
    const size_t q8 = ((size_t)(K / 32) * 34 + 15) / 16 * 16;
    const size_t f32 = in_mode == GEMV_IN_F32 ? (size_t)K * 4 : in_mode == GEMV_IN_F32_RMS ? (size_t)K * 8 : 0;
    return q8 > f32 ? q8 : f32;
}

// Greedy-argmax key: ordered fp32 bits above the inverted index, so the
// largest key is the largest value and, among equal values, the first index
// (std::max_element, sampler.cpp:34-36).  Same encoding as k_argmax.
__device__ __forceinline__ unsigned long long mv_key(float v, int64_t idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(uint32_t)(0x7FFFFFFF - (int32_t)idx);
}

// Batch-1 Q4_0 x Q8_0 mat-vec with the reference's summation order.
//
// Each CTA owns a contiguous range of rows (one CTA per SM).  A CTA takes at
// most half of an SM (480 threads, <= 64 registers, ~108 KB of shared memory),
// so under programmatic dependent launch the NEXT kernel's CTA is resident on
// the same SM while this one computes: its producer warp, which never waits on
// the previous kernel, streams the next matrix into its own ring meanwhile.
// The producer streams the rows through an ns-stage shared-memory ring, R
// whole rows per stage (nibbles and scales of the row-interleaved layout: one
// bulk copy).  For each stage the MV_CW dot
// warps compute the int32 block dots I(n, b) of its R x K/32 blocks (lanes over
// consecutive blocks of one row: conflict-free 16-byte reads) and store the
// terms (float(I), f32(dx) * f32(dw)) -- both exact -- in the stage's chain
// buffer; then chain warp g % MV_CH (stages rotate over the chain warps, so
// the chains of several stages run at once) runs, one lane per row, the fp32
// fma chain over the blocks in order: acc = fma(float(I), dx*dw, acc)
// (nnml_gemv_q4_0_4x4_q8_0, gemm.cpp:179-181; vcvtq_n_f32_s32(16 I, 4) is
// float(I) exactly).  The pair variant follows nnml_vec_dot_q4_0_q8_0
// (arm.cpp:633-692, the generic mul_mat of the lm head): four lanes per row,
// lane l accumulating partial dot l of even blocks and of odd blocks in two
// chains, then ((l0+l1)+(l2+l3)) of each, even plus odd.
//
// Every wait is bounded; on a timeout the kernel records an error code,
// stops its loops and (producer) waits for its copies in flight before exit.
template <int IN, int OUT>
__global__ void __launch_bounds__(MV_THREADS, 2)
k_mv(const GemvArgs a, const MvPlan p) {
    constexpr bool PAIR = OUT == GEMV_OUT_PAIR || OUT == GEMV_OUT_LOGITS;
    constexpr int XR = XRec<PAIR>::INTS;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_abort;
    __shared__ unsigned long long s_best[MV_CH];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nb = (int)(a.K >> 5);
    const uint32_t rowb = (uint32_t)q4_row_bytes(a.K);   // bytes per weight row (nibbles, then scales)
    const uint32_t scol = (uint32_t)(a.K >> 1);           // scales' offset in a row
    constexpr int US = OUT == GEMV_OUT_SWIGLU ? 2 : 1;   // SwiGLU rows come in (gate, up) pairs
    const int64_t units = a.N / US;
    const int64_t n0 = units * blockIdx.x / gridDim.x * US, n1 = units * (blockIdx.x + 1) / gridDim.x * US;
    const int R = p.R;
    const int nst = (int)((n1 - n0 + R - 1) / R);
    uint64_t * full = reinterpret_cast<uint64_t *>(smem + p.bar_off);
    uint64_t * empty = full + p.ns;
    uint64_t * done = empty + p.ns;
    uint64_t * freeb = done + p.ncb;
    int * xs = reinterpret_cast<int *>(smem + p.xs_off);
    uint8_t * cbase = smem + p.cb_off;
    if (tid == 0) {
        for (int i = 0; i < p.ns; ++i) { alb_mbar_init(&full[i], 1); alb_mbar_init(&empty[i], MV_CW); }
        for (int i = 0; i < p.ncb; ++i) { alb_mbar_init(&done[i], MV_CW); alb_mbar_init(&freeb[i], 1); }
        s_abort = 0;
        alb_mbar_fence_init();
    }
    if (tid < MV_CH) s_best[tid] = 0ull;
    __syncthreads();
    // the next kernel may launch now (and start its own weight stream); it waits
    // for this grid's completion before it reads anything this grid writes
    alb_pdl_trigger();

    if (warp == MV_PW) {
        // ------------------------------------------------ producer warp
        if (lane == 0) {
            int g = 0, slot = 0, round = 0;
            for (; g < nst; ++g) {
                if (round > 0 && !alb_mbar_wait(&empty[slot], (uint32_t)((round - 1) & 1))) {
                    atomicExch(a.err, ALB_DEVERR_MBAR_TIMEOUT);
                    s_abort = 1;
                    break;
                }
                const int64_t r0 = n0 + (int64_t)g * R;
                const uint32_t bytes = (uint32_t)((n1 - r0) < R ? (n1 - r0) : R) * rowb;
                alb_mbar_expect_tx(&full[slot], bytes);
                alb_bulk_g2s(smem + (size_t)slot * p.stage_bytes, a.W + r0 * rowb, bytes, &full[slot]);
                if (++slot == p.ns) { slot = 0; ++round; }
            }
            // never exit with copies in flight
            for (int j = g - p.ns < 0 ? 0 : g - p.ns; j < g; ++j)
                alb_mbar_wait(&full[j % p.ns], (uint32_t)((j / p.ns) & 1));
        }
        return;
    }

    // ------------------------------------- dot and chain warps: the input records
    if constexpr (IN == GEMV_IN_F32_RMS) {
        // the norm weights do not depend on the previous kernel (the prologue's
        // first barrier orders these stores before their use)
        float * wf = reinterpret_cast<float *>(cbase) + a.K;
        if ((reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0)
            mv_stage16(reinterpret_cast<uint4 *>(wf), reinterpret_cast<const uint4 *>(a.norm_w), (int)(a.K / 4));
        else
            for (int i = tid; i < (int)a.K; i += MV_NT) wf[i] = a.norm_w[i];
    }
    alb_pdl_wait();
    mv_prologue<IN, PAIR>(a, xs, nb, reinterpret_cast<uint4 *>(cbase));

    if (warp < MV_CW) {
        // ---------------------------------------------------- block-dot warps
        // This warp's lanes own blocks b = 32 * group + lane for the whole launch
        // (their Q8_0 records stay in registers); each stage, the m warps of the
        // group take its rows j, j + m, ..., MV_RU rows per iteration.
        // dot warp w: block group w % nbg, row phase w / nbg among the
        // ceil((MV_CW - group) / nbg) warps of that group (every group gets one:
        // nb <= 32 * MV_CW)
        const int nbg = (nb + 31) >> 5;
        const int bg = warp % nbg, jr = warp / nbg, m = (MV_CW - bg + nbg - 1) / nbg;
        const int b = bg * 32 + lane;
        const bool valid = b < nb;
        int4 lo = make_int4(0, 0, 0, 0), hi = lo;
        int asum = 0, sg0 = 0, sg1 = 0, sg2 = 0, sg3 = 0;
        float dxv = 0.0f;
        if (valid) {
            const int * rec = xs + b * XR;
            lo = *reinterpret_cast<const int4 *>(rec);
            hi = *reinterpret_cast<const int4 *>(rec + 4);
            dxv = __int_as_float(rec[8]);
            if constexpr (!PAIR) {
                asum = rec[9];
            } else {
                const int4 ds = *reinterpret_cast<const int4 *>(rec + 8);    // d, sum, s0, s1
                const int2 s23 = *reinterpret_cast<const int2 *>(rec + 12);  // s2, s3
                sg0 = ds.z; sg1 = ds.w; sg2 = s23.x; sg3 = s23.y;
            }
        }
        // fp16 bits of dx for the exact mixed-precision product dx * dw
        const unsigned short dxh = __half_as_ushort(__float2half_rn(dxv));
        const uint32_t wofs = 16u * (uint32_t)b, sofs = scol + 2u * (uint32_t)b;
        const int n_rows = (int)(n1 - n0);
        int slot = 0, cbi = 0, ring_round = 0, chain_round = 0;
        for (int g = 0; g < nst; ++g) {
            if (*reinterpret_cast<volatile int *>(&s_abort)) break;
            bool ok = alb_mbar_wait(&full[slot], (uint32_t)(ring_round & 1));
            if (ok && chain_round > 0) ok = alb_mbar_wait(&freeb[cbi], (uint32_t)((chain_round - 1) & 1));
            if (!ok) {
                if (lane == 0) atomicExch(a.err, ALB_DEVERR_MBAR_TIMEOUT);
                s_abort = 1;
                break;
            }
            const int rb = g * R;
            const int rg = n_rows - rb < R ? n_rows - rb : R;
            const uint8_t * stg = smem + (uint32_t)slot * p.stage_bytes;
            uint8_t * cb = cbase + (uint32_t)cbi * p.cb_bytes;
            if (valid) {
                for (int r = jr; r < rg; r += MV_RU * m) {
                    uint4 w[MV_RU];
                    unsigned short dwb[MV_RU];
#pragma unroll
                    for (int k = 0; k < MV_RU; ++k) {
                        if (r + k * m < rg) {
                            const uint8_t * row = stg + (uint32_t)(r + k * m) * rowb;
                            w[k] = *reinterpret_cast<const uint4 *>(row + wofs);
                            dwb[k] = *reinterpret_cast<const unsigned short *>(row + sofs);
                        }
                    }
#pragma unroll
                    for (int k = 0; k < MV_RU; ++k) {
                        const int rk = r + k * m;
                        if (rk < rg) {
                            const float s = alb_mul_f16_exact(dxh, dwb[k]);   // f32(dx) * f32(dw), exact
                            if constexpr (!PAIR) {
                                const int I = q4q8_dot_fast(w[k], lo, hi, asum);
                                *reinterpret_cast<float2 *>(cb + (uint32_t)rk * p.cbp + 8u * (uint32_t)b) =
                                    make_float2(alb_i2f_small(I), s);
                                if constexpr (OUT == GEMV_OUT_DOTS) a.dots[(n0 + rb + rk) * nb + b] = I;
                            } else {
                                const uint32_t wv[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
                                const int lov[4] = {lo.x, lo.y, lo.z, lo.w}, hiv[4] = {hi.x, hi.y, hi.z, hi.w};
                                const int sg[4] = {sg0, sg1, sg2, sg3};
                                int pl[4];
#pragma unroll
                                for (int l = 0; l < 4; ++l) {
                                    int lo_s = 0, hi_s = 0;
                                    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(lo_s) : "r"(wv[l] & 0x0F0F0F0Fu), "r"(lov[l]));
                                    asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(hi_s) : "r"(wv[l] & 0xF0F0F0F0u), "r"(hiv[l]));
                                    pl[l] = lo_s + (hi_s >> 4) - 8 * sg[l];   // hi_s = 16 * sum(hi * a): exact shift
                                }
                                float * T = reinterpret_cast<float *>(cb + (uint32_t)rk * p.cbp) + 4 * b;
                                float * S = reinterpret_cast<float *>(cb + (uint32_t)R * p.cbp + (uint32_t)rk * p.cbs) + b;
                                if ((nb & 1) && b == nb - 1) {
                                    // scalar tail of an odd block count (arm.cpp:675-691): sumi, dw, dx
                                    *reinterpret_cast<float4 *>(T) = make_float4(
                                        alb_i2f_small(pl[0] + pl[1] + pl[2] + pl[3]), alb_h2f_bits(dwb[k]), 0.0f, 0.0f);
                                    *S = dxv;
                                } else {
                                    *reinterpret_cast<float4 *>(T) = make_float4(alb_i2f_small(pl[0]), alb_i2f_small(pl[1]),
                                                                                 alb_i2f_small(pl[2]), alb_i2f_small(pl[3]));
                                    *S = s;
                                }
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) { alb_mbar_arrive(&empty[slot]); alb_mbar_arrive(&done[cbi]); }
            if (++slot == p.ns) { slot = 0; ++ring_round; }
            if (++cbi == MV_CH) { cbi = 0; ++chain_round; }
        }
        return;
    }

    // ---------------------------------------------------------- chain warps
    // Chain warp cw takes the stages g = cw, cw + MV_CH, ... (chain buffer cw),
    // all their rows, in passes of RC rows (one lane per row; four for the pair chain).
    const int cw = warp - MV_CW;
    unsigned long long best = 0ull;   // LOGITS: this lane's best key
    for (int g = cw; g < nst; g += MV_CH) {
        const int cbi = cw;   // g % MV_CH
        if (*reinterpret_cast<volatile int *>(&s_abort)) break;
        if (!alb_mbar_wait(&done[cbi], (uint32_t)((g / MV_CH) & 1))) {
            if (lane == 0) atomicExch(a.err, ALB_DEVERR_MBAR_TIMEOUT);
            s_abort = 1;
            break;
        }
        const int64_t r0 = n0 + (int64_t)g * R;
        const int rg = (int)((n1 - r0) < R ? (n1 - r0) : R);
        const uint8_t * cb = cbase + (size_t)cbi * p.cb_bytes;
        if constexpr (!PAIR) {
            float accs[2];   // R <= 64: at most two passes of 32 rows
#pragma unroll
            for (int ps = 0; ps < 2; ++ps) {
                // acc = fma(float(I), f32(dx) * f32(dw), acc), blocks in order
                const int r = ps * 32 + lane;
                float acc = 0.0f;
                if (r < rg) {
                    const float4 * e = reinterpret_cast<const float4 *>(cb + (size_t)r * p.cbp);
                    int b = 0;
#pragma unroll 8
                    for (; b + 1 < nb; b += 2) {
                        const float4 v = e[b >> 1];
                        acc = __fmaf_rn(v.x, v.y, acc);
                        acc = __fmaf_rn(v.z, v.w, acc);
                    }
                    if (b < nb) {
                        const float2 v = reinterpret_cast<const float2 *>(e)[b];
                        acc = __fmaf_rn(v.x, v.y, acc);
                    }
                }
                accs[ps] = acc;
            }
            __syncwarp();
            if (lane == 0) alb_mbar_arrive(&freeb[cbi]);   // the terms are in registers now
#pragma unroll
            for (int ps = 0; ps < 2; ++ps) {
                const int r = ps * 32 + lane;
                const float acc = accs[ps];
                if constexpr (OUT == GEMV_OUT_SWIGLU) {
                    // passes hold 32 rows: gate row r (even) and up row r + 1 share the warp
                    const float up = __shfl_down_sync(0xffffffffu, acc, 1);
                    if (r < rg && !(r & 1)) a.y[(r0 + r) >> 1] = alb_swiglu1(acc, up);
                } else {
                    if (r < rg && a.y) {
                        const int64_t n = r0 + r;
                        a.y[n] = a.residual ? __fadd_rn(acc, a.residual[n]) : acc;
                    }
                }
            }
        } else {
            float sums[2];   // R <= 16: at most two passes of 8 rows
#pragma unroll
            for (int ps = 0; ps < 2; ++ps) {
                const int rr = ps * 8 + (lane >> 2), l = lane & 3;
                const bool mine = rr < rg;
                float sv0 = 0.0f, sv1 = 0.0f;
                float tail = 0.0f;
                if (mine) {
                    const float * T = reinterpret_cast<const float *>(cb + (size_t)rr * p.cbp) + l;
                    const float * S = reinterpret_cast<const float *>(cb + (size_t)R * p.cbp + (size_t)rr * p.cbs);
                    int b = 0;
#pragma unroll 8
                    for (; b + 1 < nb; b += 2) {
                        sv0 = __fmaf_rn(T[4 * b], S[b], sv0);
                        sv1 = __fmaf_rn(T[4 * b + 4], S[b + 1], sv1);
                    }
                    if (b < nb) {   // odd block count: ((sumi * dw) * dx), added after the vector sum
                        const float * Tt = T - l + 4 * b;
                        tail = __fmul_rn(__fmul_rn(Tt[0], Tt[1]), S[b]);
                    }
                }
                // vaddvq_f32 = (l0 + l1) + (l2 + l3), then sumv0 + sumv1 (arm.cpp:671)
                float a0 = __fadd_rn(sv0, __shfl_xor_sync(0xffffffffu, sv0, 1));
                a0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 2));
                float a1 = __fadd_rn(sv1, __shfl_xor_sync(0xffffffffu, sv1, 1));
                a1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 2));
                float sum = __fadd_rn(a0, a1);
                if (nb & 1) sum = __fadd_rn(sum, tail);
                sums[ps] = sum;
            }
            __syncwarp();
            if (lane == 0) alb_mbar_arrive(&freeb[cbi]);
#pragma unroll
            for (int ps = 0; ps < 2; ++ps) {
                const int rr = ps * 8 + (lane >> 2), l = lane & 3;
                if (rr < rg && l == 0) {
                    const int64_t n = r0 + rr;
                    const float sum = sums[ps];
                    if (a.y) a.y[n] = sum;
                    if constexpr (OUT == GEMV_OUT_LOGITS) {
                        if (sum == sum) {
                            const unsigned long long k = mv_key(sum, a.idx_base + n);
                            best = k > best ? k : best;
                        }
                    }
                }
            }
        }
    }
    if constexpr (OUT == GEMV_OUT_LOGITS) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0) s_best[cw] = best;
        asm volatile("bar.sync 2, %0;" :: "n"(MV_CH * 32) : "memory");
        if (cw == 0 && lane == 0) {
            unsigned long long m = 0ull;
#pragma unroll
            for (int w = 0; w < MV_CH; ++w) m = s_best[w] > m ? s_best[w] : m;
            if (m) atomicMax(a.key, m);
            if (a.next) {
                __threadfence();
                if (atomicAdd(a.ticket, 1) == (int)gridDim.x - 1) {
                    __threadfence();
                    const unsigned long long k = atomicOr(a.key, 0ull);
                    if (k == 0ull) atomicExch(a.err, ALB_DEVERR_BAD_TOKEN);
                    *a.next = k ? 0x7FFFFFFF - (int32_t)(k & 0xFFFFFFFFull) : 0;
                    *a.ticket = 0;
                }
            }
        }
    }
}

// odd multiple of 16 >= x (distinct 16-byte bank groups for rows read together)
static inline uint32_t mv_odd16(uint32_t x) {
    uint32_t r = (x + 15) & ~15u;
    if (((r >> 4) & 1) == 0) r += 16;
    return r;
}

// Shared-memory plan: stages of about `stage_target` bytes of whole rows (one
// bulk copy each: large copies stream at full HBM rate, small ones are limited
// by the per-copy cost), one chain buffer per chain warp, and as many stages
// (2..8) as fit the budget (about half an SM's shared memory, so that the next
// launch's CTA fits beside this one and prefetches its own weights).
static MvPlan mv_plan(int64_t K, bool pair, int in_mode, int budget, int stage_target) {
    const int64_t nb = K / 32;
    const int64_t row_bytes = q4_row_bytes(K);
    const int rmax = pair ? 16 : 64;   // two chain passes of 8 (pair) or 32 rows
    int R = (int)(stage_target / row_bytes);
    if (R > rmax) R = rmax;
    if (R < 2) R = 2;
    R &= ~1;
    MvPlan p{};
    for (;;) {
        p.R = R;
        p.RC = pair ? 8 : 32;
        p.ns = 2;
        p.ncb = MV_CH;
        p.stage_bytes = (uint32_t)(R * row_bytes);
        // chain entries per (row, block): (float(I), dx * dw), or for the pair
        // chain the four float partial dots [R][nb][4] and dx * dw [R][nb]
        p.cbp = mv_odd16((uint32_t)(nb * (pair ? 16 : 8)));
        if (pair) {
            uint32_t words = (uint32_t)nb;
            if ((words & 1) == 0) words += 1;
            p.cbs = words * 4;
            p.cb_bytes = ((uint32_t)R * p.cbp + (uint32_t)R * p.cbs + 15) & ~15u;
        } else {
            p.cbs = 0;
            p.cb_bytes = (uint32_t)R * p.cbp;
        }
        uint32_t region = (uint32_t)p.ncb * p.cb_bytes;
        const uint32_t stg = (uint32_t)gemv_stage_bytes(K, in_mode);
        if (stg > region) region = stg;
        const uint32_t xsb = (uint32_t)(nb * (pair ? XRec<true>::INTS : XRec<false>::INTS) * 4);
        const uint32_t fixed = ((region + 127) & ~127u) + ((xsb + 127) & ~127u) + 8 * 2 * (6 + p.ncb);
        while (p.ns < 8 && (int)(fixed + (uint32_t)(p.ns + 1) * p.stage_bytes) <= budget) ++p.ns;
        p.cb_off = (uint32_t)p.ns * p.stage_bytes;
        p.xs_off = p.cb_off + ((region + 127) & ~127u);
        p.bar_off = p.xs_off + ((xsb + 127) & ~127u);
        p.smem = p.bar_off + 8 * 2 * (p.ns + p.ncb);
        if ((int)p.smem <= budget || R <= 2) break;
        R = (R - 2) & ~1;
        if (R < 2) R = 2;
    }
    return p;
}

// Tuning knobs (read once per process): ALB_MV_SMEM_KB (shared-memory budget
// of a CTA, default 108: two CTAs per SM), ALB_MV_STAGE_KB (target stage size,
// default 32), ALB_MV_CPS (CTAs per SM of a launch, default 1: the other half
// of each SM is for the next launch).
static int mv_knob(const char * name, int dflt) {
    const char * v = getenv(name);
    return v && atoi(v) > 0 ? atoi(v) : dflt;
}

template <int IN, int OUT>
static cudaError_t launch_mv_t(const GemvArgs & a, cudaStream_t stream) {
    constexpr bool PAIR = OUT == GEMV_OUT_PAIR || OUT == GEMV_OUT_LOGITS;
    static const int budget_kb = mv_knob("ALB_MV_SMEM_KB", 108);
    static const int stage_kb = mv_knob("ALB_MV_STAGE_KB", 32);
    const MvPlan p = mv_plan(a.K, PAIR, IN, a.smem_budget > 0 ? a.smem_budget : budget_kb * 1024, stage_kb * 1024);
    auto kern = k_mv<IN, OUT>;
    cudaError_t e = ensure_smem(kern, p.smem);
    if (e != cudaSuccess) return e;
    const int64_t units = OUT == GEMV_OUT_SWIGLU ? a.N / 2 : a.N;
    static const int cps = mv_knob("ALB_MV_CPS", 1);
    int64_t grid = a.ctas > 0 ? a.ctas : (int64_t)alb_sm_count() * cps;
    if (grid > units) grid = units;
    if (grid < 1) grid = 1;
    return alb_launch(kern, dim3((unsigned)grid), dim3(MV_THREADS), p.smem, stream, a.pdl, a, p);
}

template <int IN>
static cudaError_t dispatch_out(const GemvArgs & a, cudaStream_t s) {
    switch (a.out_mode) {
        case GEMV_OUT_PLAIN: return launch_mv_t<IN, GEMV_OUT_PLAIN>(a, s);
        case GEMV_OUT_SWIGLU: return launch_mv_t<IN, GEMV_OUT_SWIGLU>(a, s);
        case GEMV_OUT_DOTS: return launch_mv_t<IN, GEMV_OUT_DOTS>(a, s);
        case GEMV_OUT_PAIR: return launch_mv_t<IN, GEMV_OUT_PAIR>(a, s);
        case GEMV_OUT_LOGITS: return launch_mv_t<IN, GEMV_OUT_LOGITS>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(const GemvArgs & a_in, cudaStream_t s) {
    GemvArgs a = a_in;
    if (!a.err) a.err = device_error_ptr();
    if (!a.err) return cudaErrorMemoryAllocation;
    // K <= 12288 (the C ABI's limit; the dot warps would take up to 32 * 32 * MV_CW)
    if (a.K % 32 != 0 || a.K <= 0 || a.N <= 0 || a.K > 12288 || a.N >= ((int64_t)1 << 30))
        return cudaErrorInvalidValue;
    // bulk copies: 16-byte aligned sources (row strides K/2 and pitch*2 are multiples of 16)
    if (reinterpret_cast<uintptr_t>(a.W) & 15) return cudaErrorInvalidValue;   // bulk-copy source alignment
    if (a.out_mode == GEMV_OUT_SWIGLU && a.N % 2 != 0) return cudaErrorInvalidValue;
    if (a.out_mode == GEMV_OUT_SWIGLU && !a.y) return cudaErrorInvalidValue;
    if (a.out_mode == GEMV_OUT_LOGITS && (!a.key || (a.next && !a.ticket))) return cudaErrorInvalidValue;
    if (a.out_mode == GEMV_OUT_DOTS && !a.dots) return cudaErrorInvalidValue;
    switch (a.in_mode) {
        case GEMV_IN_Q8: return dispatch_out<GEMV_IN_Q8>(a, s);
        case GEMV_IN_F32: return dispatch_out<GEMV_IN_F32>(a, s);
        case GEMV_IN_F32_RMS: return dispatch_out<GEMV_IN_F32_RMS>(a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace alb

// ================================================================ C ABI
using namespace alb;

extern "C" size_t alb_q4_0_gpu_bytes(int64_t N, int64_t K) { return q4_gpu_bytes(N, K); }
extern "C" size_t alb_q4_0_row_bytes(int64_t K) { return (K > 0 && K % 32 == 0) ? (size_t)q4_row_bytes(K) : 0; }

extern "C" int alb_repack_q4_0(void * dst, const void * src, int64_t N, int64_t K, void * stream) {
    ALB_CHECK_ARG(dst && src && N > 0 && K > 0 && K % 32 == 0);
    const int64_t nbk = N * (K / 32);
    k_repack_q4_0<<<(unsigned)((nbk + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (uint8_t *)dst, (const uint8_t *)src, nbk, K / 32, q4_scale_pitch(K), q4_row_bytes(K));
    ALB_CUDA_TRY(cudaGetLastError());
    return ALB_OK;
}

extern "C" int alb_unpack_q4_0(void * dst, const void * src, int64_t N, int64_t K, void * stream) {
    ALB_CHECK_ARG(dst && src && N > 0 && K > 0 && K % 32 == 0);
    const int64_t nbk = N * (K / 32);
    k_unpack_q4_0<<<(unsigned)((nbk + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (uint8_t *)dst, (const uint8_t *)src, nbk, K / 32, q4_row_bytes(K));
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
    a.W = (const uint8_t *)W; a.N = N; a.K = K;
    a.in_mode = GEMV_IN_Q8; a.x = xq;
    a.out_mode = GEMV_OUT_PLAIN; a.y = y; a.residual = residual;
    a.pdl = true;
    ALB_CUDA_TRY(launch_gemv(a, (cudaStream_t)stream));
    return ALB_OK;
}

extern "C" int alb_mul_mat_q4_0_q8_0(const void * W, const void * xq, float * y, int64_t N, int64_t K, void * stream) {
    ALB_CHECK_ARG(W && xq && y && N > 0 && K > 0 && K % 32 == 0 && K <= 12288);
    GemvArgs a;
    a.W = (const uint8_t *)W; a.N = N; a.K = K;
    a.in_mode = GEMV_IN_Q8; a.x = xq;
    a.out_mode = GEMV_OUT_PAIR; a.y = y;
    a.pdl = true;
    ALB_CUDA_TRY(launch_gemv(a, (cudaStream_t)stream));
    return ALB_OK;
}

extern "C" int alb_gemv_q4_0_q8_0_block_dots(const void * W, const void * xq, int32_t * I, int64_t N, int64_t K,
                                             void * stream) {
    ALB_CHECK_ARG(W && xq && I && N > 0 && K > 0 && K % 32 == 0 && K <= 12288);
    GemvArgs a;
    a.W = (const uint8_t *)W; a.N = N; a.K = K;
    a.in_mode = GEMV_IN_Q8; a.x = xq;
    a.out_mode = GEMV_OUT_DOTS; a.dots = I; a.y = nullptr;
    ALB_CUDA_TRY(launch_gemv(a, (cudaStream_t)stream));
    return ALB_OK;
}
