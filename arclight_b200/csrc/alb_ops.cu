// Elementwise / attention / sampling kernels of the Qwen3 decode/prefill path
// (sm_100a).  Reference semantics cited per kernel.
#include <cfloat>
#include <cmath>

#include "alb_common.cuh"
#include "alb_internal.h"
#include "alb_q4_dev.cuh"

namespace alb {

// ------------------------------------------------------------------ embedding
// GET_ROWS on the Q4_0 token table (ops.cpp:12-52, dequantize_row_q4_0
// types.cpp:337-350): x[t][j] = (q - 8) * d.  One thread per 32-value block.
// The first kernel of a forward pass also clears the greedy-argmax key that
// the lm head of this pass accumulates into (key may be null).
__global__ void k_embed_q4_0(const uint8_t * __restrict__ W, const int32_t * __restrict__ tokens, int T, int64_t E,
                             int64_t vocab, float * __restrict__ x, int * err, unsigned long long * key) {
    const int64_t nb = E / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * nb) return;
    const int t = (int)(i / nb), b = (int)(i - (int64_t)t * nb);
    alb_pdl_wait();
    if (key && i == 0) *key = 0ull;
    int32_t tok = tokens[t];
    if (tok < 0 || tok >= vocab) { atomicExch(err, 3); tok = 0; }
    const uint8_t * row = W + (size_t)tok * q4_row_bytes(E);   // row-interleaved GPU layout
    const uint4 v = *reinterpret_cast<const uint4 *>(row + 16 * b);
    const float d = alb_h2f(reinterpret_cast<const uint16_t *>(row + E / 2)[b]);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float * o = x + (size_t)t * E + 32 * b;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int byte = (w[k] >> (8 * j)) & 0xFF;
            o[4 * k + j] = (float)((byte & 0x0F) - 8) * d;
            o[16 + 4 * k + j] = (float)((byte >> 4) - 8) * d;
        }
    alb_pdl_trigger();
}

// ------------------------------------------------- QK-norm + RoPE + KV store
// Per token t and head: Q heads get RMSNorm(128)*q_norm (qwen3.cpp:215-217,
// ops.cpp:680-724) then NEOX RoPE at pos0+t (ops.cpp:830-938) using the host
// cos/sin table (nnml_rope_cache_init, ops.cpp:759-771); K heads likewise with
// k_norm and are stored fp32->fp16 (RNE) into the K cache row pos0+t
// (set_rows, ops.cpp:135-181); V heads are stored as is.
// Block = 128 threads (one per dimension), grid = (Hq + 2*Hkv, T).
__global__ void __launch_bounds__(128)
k_qk_norm_rope_kv(const float * __restrict__ qkv, int64_t qkv_stride, int Hq, int Hkv,
                  const float * __restrict__ qn_w, const float * __restrict__ kn_w, float eps,
                  const float2 * __restrict__ rope, int32_t pos0, const int32_t * __restrict__ pos_dev,
                  float * __restrict__ q_out, uint16_t * __restrict__ kc, uint16_t * __restrict__ vc,
                  int64_t kv_row) {
    const int head = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
    const int lane = d & 31, warp = d >> 5;
    alb_pdl_wait();
    const int32_t pos = (pos_dev ? pos_dev[0] : pos0) + t;
    const float * src = qkv + (size_t)t * qkv_stride;
    __shared__ float buf[128];
    __shared__ double red[4];
    if (head >= Hq + Hkv) {   // V head: plain fp16 store
        const int hv = head - Hq - Hkv;
        vc[(size_t)pos * kv_row + hv * 128 + d] = alb_f2h(src[(Hq + Hkv) * 128 + hv * 128 + d]);
        alb_pdl_trigger();
        return;
    }
    const bool is_q = head < Hq;
    const int hh = is_q ? head : head - Hq;
    const float v = src[(is_q ? 0 : Hq * 128) + hh * 128 + d];
    double s = (double)__fmul_rn(v, v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    // reference order: ((s0 + s1) + s2) + s3 over 32-lane partials of a sequential
    // double sum -- any order of 128 fp32 squares in double rounds identically
    const double tot = red[0] + red[1] + red[2] + red[3];
    const float mean = (float)(tot / 128.0);
    const float scale = 1.0f / sqrtf(__fadd_rn(mean, eps));
    const float nv = __fmul_rn(__fmul_rn(v, scale), (is_q ? qn_w : kn_w)[d]);
    buf[d] = nv;
    __syncthreads();
    float outv;
    const float2 cs = rope[(size_t)pos * 64 + (d & 63)];
    if (d < 64) outv = __fsub_rn(__fmul_rn(buf[d], cs.x), __fmul_rn(buf[d + 64], cs.y));
    else        outv = __fadd_rn(__fmul_rn(buf[d - 64], cs.y), __fmul_rn(buf[d], cs.x));
    if (is_q) q_out[((size_t)t * Hq + hh) * 128 + d] = outv;
    else      kc[(size_t)pos * kv_row + hh * 128 + d] = alb_f2h(outv);
    alb_pdl_trigger();
}

// ------------------------------------------------------------ flash attention
// nnml_compute_forward_flash_attn_ext_f16 (arm.cpp:2196-2433) for F16 K/V, one
// sequence, causal: token t (position p0 + t) attends cells [0, p0+t+1).
// Semantics (identical to the oracle's fp32 mode, independent of how the cells
// are split across CTAs): Q rounded to fp16 as the reference does
// (arm.cpp:2307); score s_c = sequential fp32 fma chain over d of K.Q, times
// scale; M = max_c s_c; p_c = v_expf(s_c - M) (the reference's NEON exp,
// arm.cpp:1757-1787); L = sum p_c and O_d = sum p_c V_cd in double; out = O/L.
// Softmax is shift invariant, so this is the reference's online softmax with
// different (and fewer) roundings.
//
// Decode splits the cells over S CTAs: k_fa_scores writes the scores and
// per-split maxima, k_fa_pv applies the global max and accumulates its split in
// double, k_fa_merge adds the S partials of each query head in split order (and
// can emit the block_q8_0 records of the result).  Prefill ubatches (T > 1, one
// split) use k_fa_prefill (token tiles over staged cells); k_fa_fused (one CTA
// per (h, t), scores in shared memory) serves single-split single-token calls.
static constexpr int FA_TICKETS = 8192;

__device__ __forceinline__ float fa_score(const uint16_t * __restrict__ krow, const float * __restrict__ qg) {
    const uint4 * kr = reinterpret_cast<const uint4 *>(krow);
    float a = 0.0f;
#pragma unroll 4
    for (int j = 0; j < 16; ++j) {
        const uint4 kv = kr[j];
        const uint32_t wd[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 kf = __half22float2(*reinterpret_cast<const __half2 *>(&wd[e]));
            const int d = 8 * j + 2 * e;
            a = __fmaf_rn(kf.x, qg[d], a);
            a = __fmaf_rn(kf.y, qg[d + 1], a);
        }
    }
    return a;
}

template <int G>
__device__ __forceinline__ void fa_load_q(const float * __restrict__ q, int Hq, int h, int t, float (*qs)[128]) {
    for (int i = threadIdx.x; i < G * 128; i += blockDim.x) {
        const int g = i / 128, d = i - g * 128;
        qs[g][d] = __half2float(__float2half_rn(q[((size_t)t * Hq + h * G + g) * 128 + d]));
    }
}

// Splits in use for n cells: at most S, at least FA_MIN_SPLIT cells each (short
// contexts use fewer CTAs and the merge adds fewer partials).  Computed on the
// device from the position, so a captured graph serves every context length.
static constexpr int FA_MIN_SPLIT = 128;
__device__ __forceinline__ int fa_splits_used(int n, int S) {
    const int m = (n + FA_MIN_SPLIT - 1) / FA_MIN_SPLIT;
    return m < 1 ? 1 : (m < S ? m : S);
}

__device__ __forceinline__ void fa_split(int n, int S, int s, int & c0, int & c1) {
    int sz = (n + S - 1) / S;
    c0 = s * sz;
    c1 = min(n, c0 + sz);
    if (c0 > n) c0 = n;
}

// Split kernels stream K and V through a shared-memory ring filled by
// cp.async (FA_NST stages of FA_CH cells, FA_NST - 1 stages in flight), so each
// CTA keeps tens of KB of HBM reads outstanding while it computes, with ~52 KB
// of shared memory: four CTAs (16 warps) per SM.  Two threads per cell, each
// with half of the G query heads.  K rows are padded to 272 B in shared memory
// so the 16-byte row reads of a quarter-warp fall in distinct banks.
static constexpr int FA_CH = 64;                           // cells per stage (two threads per cell)
static constexpr int FA_NST = 3;                           // ring stages
static constexpr int FA_KPITCH = 272;                      // bytes per staged K row
static constexpr int FA_KSTAGE = FA_CH * FA_KPITCH;        // 17,408 B
static constexpr int FA_VSTAGE = FA_CH * 256;              // 16,384 B
template <int G> __host__ __device__ constexpr int fa_gh() { return G >= 2 ? 2 : 1; }   // head halves (threads per cell)
static constexpr size_t FA_SCORES_SMEM = (size_t)FA_NST * FA_KSTAGE;
template <int G>
constexpr size_t fa_pv_smem() { return (size_t)FA_NST * (FA_VSTAGE + G * FA_CH * 4); }

__device__ __forceinline__ void fa_cp16(void * dst, const void * src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(alb_smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void fa_cp4(void * dst, const void * src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(alb_smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void fa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void fa_wait_ring() {   // all but the newest FA_NST - 2 groups have landed
    asm volatile("cp.async.wait_group %0;" :: "n"(FA_NST - 2) : "memory");
}
__device__ __forceinline__ void fa_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int G>
__global__ void __launch_bounds__(128)
k_fa_scores(const float * __restrict__ q, const uint16_t * __restrict__ kc, int Hq, int Hkv, int T, int32_t pos0,
            const int32_t * __restrict__ pos_dev, float scale, int S, int ncap, float * __restrict__ scores,
            float * __restrict__ smax) {
    extern __shared__ __align__(16) uint8_t fa_ring[];   // FA_NST x FA_CH x FA_KPITCH
    __shared__ __align__(16) float qs[G][128];
    __shared__ float red[4][G];
    const int h = blockIdx.x, t = blockIdx.y, s = blockIdx.z, tid = threadIdx.x;
    alb_pdl_wait();
    const int n = (pos_dev ? pos_dev[0] : pos0) + t + 1;
    const int Su = fa_splits_used(n, S);
    if (s >= Su) return;
    int c0, c1;
    fa_split(n, Su, s, c0, c1);
    const int64_t row = (int64_t)Hkv * 128;
    const uint16_t * kb = kc + (size_t)h * 128;
    const int nst = (c1 - c0 + FA_CH - 1) / FA_CH;
    auto issue = [&](int i) {
        if (i < nst) {
            const int cb = c0 + i * FA_CH, rows = min(FA_CH, c1 - cb);
            uint8_t * dst = fa_ring + (i % FA_NST) * FA_KSTAGE;
            for (int p = tid; p < rows * 16; p += 128) {
                const int r = p >> 4, j = p & 15;
                fa_cp16(dst + r * FA_KPITCH + j * 16, kb + (size_t)(cb + r) * row + j * 8);
            }
        }
        fa_commit();   // one group per stage, empty past the end
    };
#pragma unroll
    for (int i = 0; i < FA_NST - 1; ++i) issue(i);
    fa_load_q<G>(q, Hq, h, t, qs);
    constexpr int GH = fa_gh<G>(), GPT = G / GH;
    const int cl = tid & (FA_CH - 1), gh = tid / FA_CH;   // cell of the stage, head half
    float mx[GPT];
#pragma unroll
    for (int k = 0; k < GPT; ++k) mx[k] = -INFINITY;
    float * sc = scores + ((size_t)h * T + t) * G * ncap;
    for (int i = 0; i < nst; ++i) {
        fa_wait_ring();
        __syncthreads();   // stage i visible to all; stage i-1 consumed by all
        issue(i + FA_NST - 1);
        const int c = c0 + i * FA_CH + cl;
        if (gh < GH && c < c1) {
            const uint8_t * kr = fa_ring + (i % FA_NST) * FA_KSTAGE + cl * FA_KPITCH;
            float a[GPT];
#pragma unroll
            for (int k = 0; k < GPT; ++k) a[k] = 0.0f;
            uint4 krow[16];   // the whole K row in registers first: 16 independent shared loads
#pragma unroll
            for (int j = 0; j < 16; ++j) krow[j] = *reinterpret_cast<const uint4 *>(kr + j * 16);
#pragma unroll
            for (int j = 0; j < 16; ++j) {   // dims 8j .. 8j+7, in order (the reference's sequential chain)
                const uint4 kv = krow[j];
                const uint32_t wd[4] = {kv.x, kv.y, kv.z, kv.w};
                float kf[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&wd[e]));
                    kf[2 * e] = f.x;
                    kf[2 * e + 1] = f.y;
                }
#pragma unroll
                for (int k = 0; k < GPT; ++k) {
                    const float * qg = qs[gh * GPT + k];
                    const float4 qa = *reinterpret_cast<const float4 *>(qg + 8 * j);
                    const float4 qb = *reinterpret_cast<const float4 *>(qg + 8 * j + 4);
                    a[k] = __fmaf_rn(kf[0], qa.x, a[k]);
                    a[k] = __fmaf_rn(kf[1], qa.y, a[k]);
                    a[k] = __fmaf_rn(kf[2], qa.z, a[k]);
                    a[k] = __fmaf_rn(kf[3], qa.w, a[k]);
                    a[k] = __fmaf_rn(kf[4], qb.x, a[k]);
                    a[k] = __fmaf_rn(kf[5], qb.y, a[k]);
                    a[k] = __fmaf_rn(kf[6], qb.z, a[k]);
                    a[k] = __fmaf_rn(kf[7], qb.w, a[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < GPT; ++k) {
                const float v = __fmul_rn(a[k], scale);
                sc[(size_t)(gh * GPT + k) * ncap + c] = v;
                mx[k] = fmaxf(mx[k], v);
            }
        }
    }
    fa_wait_all();
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float m = alb_warp_max(g / GPT == gh ? mx[g % GPT] : -INFINITY);
        if (lane == 0) red[warp][g] = m;
    }
    __syncthreads();
    if (tid < G) {
        const int g = tid;
        smax[(((size_t)h * T + t) * S + s) * G + g] = fmaxf(fmaxf(red[0][g], red[1][g]), fmaxf(red[2][g], red[3][g]));
    }
    alb_pdl_trigger();
}

// V rows and the split's scores stream through the ring; each stage, warp w
// owns cells w, w+4, .. of the stage: its lanes turn those cells' scores into
// p = v_expf(s - M) (L in double) and p * 2^1008 as a double, then the warp
// accumulates the cells with lane owning dims 4*lane .. 4*lane+3:
// O += (p * 2^1008) * (v * 2^-1008), the V element's bits placed in a double
// with no conversion instruction (the product is p * v exactly, as fma(p, v, O)
// in double).  One CTA barrier per stage (the ring), none between the phases.
template <int G>
__global__ void __launch_bounds__(128)
k_fa_pv(const uint16_t * __restrict__ vc, int Hq, int Hkv, int T, int32_t pos0, const int32_t * __restrict__ pos_dev,
        int S, int ncap, const float * __restrict__ scores, const float * __restrict__ smax, double * __restrict__ part,
        float * __restrict__ out) {
    extern __shared__ __align__(16) uint8_t fa_ring[];   // FA_NST x (V rows [FA_CH][256 B] + scores [G][FA_CH])
    __shared__ __align__(16) double pd[FA_CH][G];
    __shared__ float M[G];
    __shared__ double Lred[4][G];
    const int h = blockIdx.x, t = blockIdx.y, s = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int STAGE = FA_VSTAGE + G * FA_CH * 4;
    alb_pdl_wait();
    const int n = (pos_dev ? pos_dev[0] : pos0) + t + 1;
    const int Su = fa_splits_used(n, S);
    if (s >= Su) return;
    int c0, c1;
    fa_split(n, Su, s, c0, c1);
    const int64_t row = (int64_t)Hkv * 128;
    const uint16_t * vb = vc + (size_t)h * 128;
    const float * sc = scores + ((size_t)h * T + t) * G * ncap;
    const int nst = (c1 - c0 + FA_CH - 1) / FA_CH;
    auto issue = [&](int i) {
        if (i < nst) {
            const int cb = c0 + i * FA_CH, rows = min(FA_CH, c1 - cb);
            uint8_t * dst = fa_ring + (i % FA_NST) * STAGE;
            for (int p = tid; p < rows * 16; p += 128) {
                const int r = p >> 4, j = p & 15;
                fa_cp16(dst + r * 256 + j * 16, vb + (size_t)(cb + r) * row + j * 8);
            }
            if (tid < rows) {
                float * sdst = reinterpret_cast<float *>(dst + FA_VSTAGE);
#pragma unroll
                for (int g = 0; g < G; ++g) fa_cp4(sdst + g * FA_CH + tid, sc + (size_t)g * ncap + cb + tid);
            }
        }
        fa_commit();
    };
#pragma unroll
    for (int i = 0; i < FA_NST - 1; ++i) issue(i);
    if (tid < G) {
        float m = -INFINITY;
        for (int k = 0; k < Su; ++k) m = fmaxf(m, smax[(((size_t)h * T + t) * S + k) * G + tid]);
        M[tid] = m;
    }
    constexpr int GL = G >= 2 ? G / 2 : 1;   // heads per lane in the softmax phase
    double L[GL], O[G][4];
#pragma unroll
    for (int k = 0; k < GL; ++k) L[k] = 0.0;
#pragma unroll
    for (int g = 0; g < G; ++g) O[g][0] = O[g][1] = O[g][2] = O[g][3] = 0.0;
    for (int i = 0; i < nst; ++i) {
        fa_wait_ring();
        __syncthreads();   // stage i visible; stage i-1 consumed by all; M visible
        issue(i + FA_NST - 1);
        const uint8_t * stg = fa_ring + (i % FA_NST) * STAGE;
        const int rows = min(FA_CH, c1 - (c0 + i * FA_CH));
        {   // softmax numerators of the rows this warp accumulates (lane: row, head half)
            const float * ss = reinterpret_cast<const float *>(stg + FA_VSTAGE);
            const int r = warp + 4 * (lane & 15), lh = lane >> 4;
#pragma unroll
            for (int k = 0; k < GL; ++k) {
                const int g = lh * GL + k;
                if (g < G) {
                    double v = 0.0;
                    if (r < rows) {
                        const float p = alb_ref_expf(__fsub_rn(ss[g * FA_CH + r], M[g]));
                        L[k] += (double)p;
                        v = (double)p * 0x1p1008;
                    }
                    pd[r][g] = v;
                }
            }
        }
        __syncwarp();
        // 16 rows per pass (4 per warp, loads first); rows past the stage's end
        // have p = 0 and finite (possibly stale) V bits, so they add exact zeros.
        for (int r0 = 0; r0 < rows; r0 += 16) {
            uint2 vv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                vv[u] = *reinterpret_cast<const uint2 *>(stg + (r0 + warp + 4 * u) * 256 + lane * 8);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int r = r0 + warp + 4 * u;
                const double v0 = alb_h2d_bits(vv[u].x & 0xFFFFu), v1 = alb_h2d_bits(vv[u].x >> 16);
                const double v2 = alb_h2d_bits(vv[u].y & 0xFFFFu), v3 = alb_h2d_bits(vv[u].y >> 16);
                double p[G];
                if constexpr (G % 2 == 0) {
#pragma unroll
                    for (int g = 0; g < G; g += 2) {
                        const double2 pp = *reinterpret_cast<const double2 *>(&pd[r][g]);
                        p[g] = pp.x;
                        p[g + 1] = pp.y;
                    }
                } else {
#pragma unroll
                    for (int g = 0; g < G; ++g) p[g] = pd[r][g];
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    O[g][0] = fma(p[g], v0, O[g][0]);
                    O[g][1] = fma(p[g], v1, O[g][1]);
                    O[g][2] = fma(p[g], v2, O[g][2]);
                    O[g][3] = fma(p[g], v3, O[g][3]);
                }
            }
        }
    }
    fa_wait_all();
    __syncthreads();   // the ring is free: it holds the per-warp O partials now
    double (*ored)[G][128] = reinterpret_cast<double (*)[G][128]>(fa_ring);   // [4][G][128]
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const double l = alb_warp_sum_d(g / GL == (lane >> 4) ? L[g % GL] : 0.0);
        if (lane == 0) Lred[warp][g] = l;
#pragma unroll
        for (int e = 0; e < 4; ++e) ored[warp][g][4 * lane + e] = O[g][e];
    }
    __syncthreads();
    double Ls[G], Os[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        Ls[g] = ((Lred[0][g] + Lred[1][g]) + Lred[2][g]) + Lred[3][g];
        Os[g] = ((ored[0][g][tid] + ored[1][g][tid]) + ored[2][g][tid]) + ored[3][g][tid];
    }
    if (S == 1) {
#pragma unroll
        for (int g = 0; g < G; ++g)
            out[((size_t)t * Hq + h * G + g) * 128 + tid] = Ls[g] > 0.0 ? __double2float_rn(Os[g] / Ls[g]) : 0.0f;
        alb_pdl_trigger();
        return;
    }
    double * pp = part + (((size_t)h * T + t) * S + s) * G * 129;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        pp[g * 129 + tid] = Os[g];
        if (tid == 0) pp[g * 129 + 128] = Ls[g];
    }
    alb_pdl_trigger();
}

// The S split partials of query head hq = h*G + g, out = O / L.  One CTA of
// 1024 threads per (hq, t): group j (threads 128j .. 128j+127, thread = dim)
// adds splits [Su*j/8, Su*(j+1)/8) of the Su in use in split order, then the 8 group sums are
// added in group order (a fixed association, the same on every call).  Warp w
// of group 0 owns dims 32w .. 32w+31 (one Q8_0 block of the output row, lane =
// dim) and, when xq is given, writes that block's block_q8_0 record
// (quantize_row_q8_0 of the fp32 result: the o_proj input).
template <int G>
__global__ void __launch_bounds__(1024)
k_fa_merge(const double * __restrict__ part, int Hq, int T, int S, int32_t pos0, const int32_t * __restrict__ pos_dev,
           float * __restrict__ out, uint8_t * __restrict__ xq) {
    constexpr int NG = 8;
    __shared__ double so[NG][128];
    __shared__ double sl[NG];
    const int hq = blockIdx.x, t = blockIdx.y, d = threadIdx.x & 127, j = threadIdx.x >> 7;
    const int h = hq / G, g = hq - h * G;
    alb_pdl_wait();
    const double * base = part + (((size_t)h * T + t) * S * G + g) * 129;   // split k at base + k*G*129
    constexpr size_t KS = (size_t)G * 129;
    const int Su = fa_splits_used((pos_dev ? pos_dev[0] : pos0) + t + 1, S);
    const int k0 = (int)((int64_t)Su * j / NG), k1 = (int)((int64_t)Su * (j + 1) / NG);
    double L = 0.0, O = 0.0;
    for (int k = k0; k < k1; ++k) { L += base[k * KS + 128]; O += base[k * KS + d]; }
    so[j][d] = O;
    if (d == 0) sl[j] = L;
    __syncthreads();
    if (j == 0) {
        double Lt = 0.0, Ot = 0.0;
#pragma unroll
        for (int i = 0; i < NG; ++i) { Lt += sl[i]; Ot += so[i][d]; }
        const float v = Lt > 0.0 ? __double2float_rn(Ot / Lt) : 0.0f;
        out[((size_t)t * Hq + hq) * 128 + d] = v;
        if (xq) {
            const int lane = d & 31, warp = d >> 5;
            int8_t q; uint16_t dh;
            q8_block_lane(v, q, dh);
            uint8_t * blk = xq + (((size_t)t * Hq + hq) * 4 + warp) * 34;
            if (lane == 0) *reinterpret_cast<uint16_t *>(blk) = dh;
            blk[2 + lane] = (uint8_t)q;
        }
    }
    alb_pdl_trigger();
}

// Prefill attention (ubatches of T > 1 tokens): one CTA per (KV head h, tile of
// TQ = 64/G tokens) computes the 64 rows (row r: token t0 + r/G, query head
// h*G + r%G) over K/V stages of 64 cells brought by cp.async (double-buffered),
// so each staged cell serves 64 rows instead of one.  Same arithmetic as the
// decode kernels: every score is the sequential fp32 fma chain over d of the
// fp16-rounded q (16 chains per thread: one cell, 16 rows); pass 1 takes the
// row maxima over each row's causal cells, pass 2 recomputes the same scores,
// forms p = v_expf(s - M) (L in double) and accumulates O += p * v in double as
// a register tile of 4 rows x 8 dims per thread, cell by cell in order (p kept
// as p * 2^1008 so the V bits enter the fma with no conversion instruction).
static constexpr int FP_R = 64;                 // rows per CTA
static constexpr int FP_CH = 64;                // cells per stage
static constexpr int FP_KPITCH = 272;           // padded K row in shared memory
static constexpr size_t FP_SMEM = (size_t)128 * FP_R * 4 + 2 * FP_CH * FP_KPITCH + 2 * FP_CH * 256 +
                                  (size_t)FP_R * FP_CH * 8;   // q^T, K x2, V x2, p: 133,120 B

// the 16 score chains of one cell (K row in shared memory) against rows
// 16*rg .. 16*rg+15 of q^T [128][FP_R]
__device__ __forceinline__ void fp_scores16(const uint8_t * __restrict__ kr, const float * __restrict__ qT, int rg,
                                            float (&a)[16]) {
#pragma unroll
    for (int k = 0; k < 16; ++k) a[k] = 0.0f;
#pragma unroll 2
    for (int j = 0; j < 16; ++j) {
        const uint4 kv = *reinterpret_cast<const uint4 *>(kr + j * 16);
        const uint32_t wd[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 kf = __half22float2(*reinterpret_cast<const __half2 *>(&wd[e]));
#pragma unroll
            for (int hlf = 0; hlf < 2; ++hlf) {
                const float kd = hlf ? kf.y : kf.x;
                const float * qd = qT + (8 * j + 2 * e + hlf) * FP_R + 16 * rg;
#pragma unroll
                for (int k4 = 0; k4 < 4; ++k4) {
                    const float4 q4 = *reinterpret_cast<const float4 *>(qd + 4 * k4);
                    a[4 * k4 + 0] = __fmaf_rn(kd, q4.x, a[4 * k4 + 0]);
                    a[4 * k4 + 1] = __fmaf_rn(kd, q4.y, a[4 * k4 + 1]);
                    a[4 * k4 + 2] = __fmaf_rn(kd, q4.z, a[4 * k4 + 2]);
                    a[4 * k4 + 3] = __fmaf_rn(kd, q4.w, a[4 * k4 + 3]);
                }
            }
        }
    }
}

template <int G>
__global__ void __launch_bounds__(256, 1)
k_fa_prefill(const float * __restrict__ q, const uint16_t * __restrict__ kc, const uint16_t * __restrict__ vc, int Hq,
             int Hkv, int T, int32_t pos0, const int32_t * __restrict__ pos_dev, float scale, float * __restrict__ out) {
    constexpr int TQ = FP_R / G;
    extern __shared__ __align__(16) uint8_t fp_sm[];
    float * qT = reinterpret_cast<float *>(fp_sm);                            // [128][FP_R]
    uint8_t * kst = fp_sm + (size_t)128 * FP_R * 4;                           // 2 x [FP_CH][FP_KPITCH]
    uint8_t * vst = kst + 2 * FP_CH * FP_KPITCH;                              // 2 x [FP_CH][256]
    double * pd = reinterpret_cast<double *>(vst + 2 * FP_CH * 256);          // [FP_R][FP_CH]
    __shared__ float Mrow[FP_R];
    __shared__ float red_m[2][FP_R];
    __shared__ double red_l[2][FP_R];
    const int h = blockIdx.x, t0 = blockIdx.y * TQ, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    alb_pdl_wait();
    const int p0 = pos_dev ? pos_dev[0] : pos0;
    const int tn = min(TQ, T - t0);                  // tokens of this tile
    const int n = p0 + t0 + tn;                      // cells seen by the tile's last token
    // q tile, transposed, rounded to fp16 (arm.cpp:2307); rows past the tile are 0
    for (int i = tid; i < FP_R * 128; i += 256) {
        const int r = i % FP_R, d = i / FP_R;
        const int tt = r / G, g = r % G;
        float v = 0.0f;
        if (tt < tn) v = __half2float(__float2half_rn(q[((size_t)(t0 + tt) * Hq + h * G + g) * 128 + d]));
        qT[d * FP_R + r] = v;
    }
    const int64_t row = (int64_t)Hkv * 128;
    const int nst = (n + FP_CH - 1) / FP_CH;
    auto issue = [&](int i, bool with_v) {
        if (i < nst) {
            const int cb = i * FP_CH, rows = min(FP_CH, n - cb);
            uint8_t * kd = kst + (i & 1) * FP_CH * FP_KPITCH;
            uint8_t * vd = vst + (i & 1) * FP_CH * 256;
            for (int p = tid; p < rows * 16; p += 256) {
                const int r = p >> 4, j = p & 15;
                const size_t src = (size_t)(cb + r) * row + (size_t)h * 128 + j * 8;
                fa_cp16(kd + r * FP_KPITCH + j * 16, kc + src);
                if (with_v) fa_cp16(vd + r * 256 + j * 16, vc + src);
            }
        }
        fa_commit();
    };
    const int cl = tid & (FP_CH - 1), rg = tid >> 6;   // score phase: cell of the stage, rows 16*rg ..
    // ---- pass 1: row maxima over the causal cells
    float mx[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) mx[k] = -INFINITY;
    issue(0, false);
    for (int i = 0; i < nst; ++i) {
        issue(i + 1, false);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();   // stage i (and q^T) visible
        const int c = i * FP_CH + cl;
        if (c < n) {
            float a[16];
            fp_scores16(kst + (i & 1) * FP_CH * FP_KPITCH + cl * FP_KPITCH, qT, rg, a);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const int tt = (16 * rg + k) / G;
                if (tt < tn && c <= p0 + t0 + tt) mx[k] = fmaxf(mx[k], __fmul_rn(a[k], scale));
            }
        }
        __syncthreads();   // buffer i & 1 consumed before stage i + 2 refills it
    }
    fa_wait_all();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const float m = alb_warp_max(mx[k]);
        if (lane == 0) red_m[warp & 1][16 * rg + k] = m;
    }
    __syncthreads();
    if (tid < FP_R) Mrow[tid] = fmaxf(red_m[0][tid], red_m[1][tid]);
    // ---- pass 2: p, L and O
    const int r4 = (tid >> 4) * 4, d8 = (tid & 15) * 8;   // P.V tile of this thread
    double L[16], O[4][8];
#pragma unroll
    for (int k = 0; k < 16; ++k) L[k] = 0.0;
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int e = 0; e < 8; ++e) O[u][e] = 0.0;
    issue(0, true);
    for (int i = 0; i < nst; ++i) {
        issue(i + 1, true);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();   // stage i visible; Mrow visible; pd free
        const int c = i * FP_CH + cl;
        float a[16];
        if (c < n) fp_scores16(kst + (i & 1) * FP_CH * FP_KPITCH + cl * FP_KPITCH, qT, rg, a);
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const int r = 16 * rg + k, tt = r / G;
            double v = 0.0;
            if (c < n && tt < tn && c <= p0 + t0 + tt) {
                const float p = alb_ref_expf(__fsub_rn(__fmul_rn(a[k], scale), Mrow[r]));
                L[k] += (double)p;
                v = (double)p * 0x1p1008;
            }
            pd[r * FP_CH + cl] = v;
        }
        __syncthreads();
        const int rows = min(FP_CH, n - i * FP_CH);
        const uint8_t * vs = vst + (i & 1) * FP_CH * 256 + d8 * 2;
        for (int cc = 0; cc < rows; ++cc) {
            const uint4 vv = *reinterpret_cast<const uint4 *>(vs + cc * 256);
            const uint32_t wd[4] = {vv.x, vv.y, vv.z, vv.w};
            double vd[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                vd[2 * e] = alb_h2d_bits(wd[e] & 0xFFFFu);
                vd[2 * e + 1] = alb_h2d_bits(wd[e] >> 16);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const double p = pd[(r4 + u) * FP_CH + cc];
#pragma unroll
                for (int e = 0; e < 8; ++e) O[u][e] = fma(p, vd[e], O[u][e]);
            }
        }
        __syncthreads();   // pd and buffer i & 1 consumed
    }
    fa_wait_all();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const double l = alb_warp_sum_d(L[k]);
        if (lane == 0) red_l[warp & 1][16 * rg + k] = l;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int r = r4 + u, tt = r / G, g = r % G;
        if (tt >= tn) continue;
        const double Ls = red_l[0][r] + red_l[1][r];
        float * o = out + ((size_t)(t0 + tt) * Hq + h * G + g) * 128 + d8;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = Ls > 0.0 ? __double2float_rn(O[u][e] / Ls) : 0.0f;
    }
    alb_pdl_trigger();
}

// One CTA per (h, t): scores of all cells in shared memory, then the same
// global-max softmax and double sums.
template <int G>
__global__ void __launch_bounds__(128)
k_fa_fused(const float * __restrict__ q, const uint16_t * __restrict__ kc, const uint16_t * __restrict__ vc, int Hq,
           int Hkv, int T, int32_t pos0, const int32_t * __restrict__ pos_dev, float scale, float * __restrict__ out) {
    extern __shared__ float fsm[];   // [G][n] scores -> probabilities
    const int h = blockIdx.x, t = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ float qs[G][128];
    __shared__ float red[4][G];
    __shared__ double Lred[4][G];
    __shared__ double ored[4][G][128];
    alb_pdl_wait();
    const int n = (pos_dev ? pos_dev[0] : pos0) + t + 1;
    fa_load_q<G>(q, Hq, h, t, qs);
    __syncthreads();
    const int64_t row = (int64_t)Hkv * 128;
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; ++g) mx[g] = -INFINITY;
    for (int c = tid; c < n; c += 128) {
        const uint16_t * krow = kc + (size_t)c * row + (size_t)h * 128;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float v = __fmul_rn(fa_score(krow, qs[g]), scale);
            fsm[(size_t)g * n + c] = v;
            mx[g] = fmaxf(mx[g], v);
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float m = alb_warp_max(mx[g]);
        if (lane == 0) red[warp][g] = m;
    }
    __syncthreads();
    float M[G];
    double L[G], O[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        M[g] = fmaxf(fmaxf(red[0][g], red[1][g]), fmaxf(red[2][g], red[3][g]));
        L[g] = 0.0; O[g][0] = O[g][1] = O[g][2] = O[g][3] = 0.0;
    }
    for (int c = tid; c < n; c += 128)
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float p = alb_ref_expf(__fsub_rn(fsm[(size_t)g * n + c], M[g]));
            fsm[(size_t)g * n + c] = p;
            L[g] += (double)p;
        }
    __syncthreads();
    for (int c = warp; c < n; c += 4) {
        const uint2 vv = *reinterpret_cast<const uint2 *>(vc + (size_t)c * row + (size_t)h * 128 + 4 * lane);
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.y));
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const double p = (double)fsm[(size_t)g * n + c];
            O[g][0] = fma(p, (double)v01.x, O[g][0]);
            O[g][1] = fma(p, (double)v01.y, O[g][1]);
            O[g][2] = fma(p, (double)v23.x, O[g][2]);
            O[g][3] = fma(p, (double)v23.y, O[g][3]);
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const double l = alb_warp_sum_d(L[g]);
        if (lane == 0) Lred[warp][g] = l;
#pragma unroll
        for (int e = 0; e < 4; ++e) ored[warp][g][4 * lane + e] = O[g][e];
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const double Ls = ((Lred[0][g] + Lred[1][g]) + Lred[2][g]) + Lred[3][g];
        const double Os = ((ored[0][g][tid] + ored[1][g][tid]) + ored[2][g][tid]) + ored[3][g][tid];
        out[((size_t)t * Hq + h * G + g) * 128 + tid] = Ls > 0.0 ? __double2float_rn(Os / Ls) : 0.0f;
    }
    alb_pdl_trigger();
}

// Workspace: [reserved FA_TICKETS ints | split maxima | scores | split partials (double)].
// Every region is written before it is read within a call (no state between calls).
struct FaLayout { size_t smax_off, scores_off, part_off, bytes; };
static FaLayout fa_layout(int Hq, int Hkv, int T, int S, int ncap) {
    const int G = Hq / Hkv;
    FaLayout l;
    l.smax_off = (size_t)FA_TICKETS * 4;
    l.scores_off = (l.smax_off + (size_t)Hkv * T * S * G * 4 + 255) & ~(size_t)255;
    l.part_off = (l.scores_off + (size_t)Hkv * T * G * ncap * 4 + 255) & ~(size_t)255;
    l.bytes = l.part_off + (size_t)Hkv * T * S * G * 129 * 8;
    return l;
}

size_t flash_attn_ws_bytes(int Hq, int Hkv, int T, int S, int ncap) {
    return fa_layout(Hq, Hkv, T, S, ncap).bytes;
}

// shared memory available for the fused kernel's score array
static constexpr size_t FA_FUSED_SMEM = 160 * 1024;

// Which kernels a call takes: the token-tiled prefill kernel (T > 1, one
// split) and the fused one-CTA kernel (one split, scores fit shared memory)
// use no workspace; every other call runs the split kernels on it.
bool flash_attn_uses_ws(int Hq, int Hkv, int T, int S, int ncap) {
    if (T > 1 && S == 1) return false;
    if (S == 1 && (size_t)(Hq / Hkv) * ncap * 4 <= FA_FUSED_SMEM) return false;
    return true;
}

template <int G>
static cudaError_t launch_fa_core(const FlashArgs & f, cudaStream_t st) {
    if (f.T > 1 && f.S == 1) {   // prefill ubatch: token tiles share the staged cells
        cudaError_t e = ensure_smem(k_fa_prefill<G>, FP_SMEM);
        if (e != cudaSuccess) return e;
        constexpr int TQ = FP_R / G;
        const dim3 grid((unsigned)f.Hkv, (unsigned)((f.T + TQ - 1) / TQ));
        return alb_launch(k_fa_prefill<G>, grid, dim3(256), FP_SMEM, st, f.pdl, f.q, f.kc, f.vc, f.Hq, f.Hkv, f.T,
                          f.pos0, f.pos_dev, f.scale, f.out);
    }
    const int n_max = f.ncap;   // cells attended by the last token at most
    if (f.S == 1 && (size_t)G * n_max * 4 <= FA_FUSED_SMEM) {
        const size_t smem = (size_t)G * n_max * 4;
        // the kernel's static shared memory counts against the 48 KiB default too
        cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void *>(k_fa_fused<G>), FA_FUSED_SMEM);
        if (e != cudaSuccess) return e;
        return alb_launch(k_fa_fused<G>, dim3((unsigned)f.Hkv, (unsigned)f.T), dim3(128), smem, st, f.pdl, f.q, f.kc,
                          f.vc, f.Hq, f.Hkv, f.T, f.pos0, f.pos_dev, f.scale, f.out);
    }
    if (!f.ws) return cudaErrorInvalidValue;
    if (f.T > 65535 || f.S > 65535) return cudaErrorInvalidValue;
    const FaLayout l = fa_layout(f.Hq, f.Hkv, f.T, f.S, f.ncap);
    uint8_t * ws = reinterpret_cast<uint8_t *>(f.ws);
    float * smax = reinterpret_cast<float *>(ws + l.smax_off);
    float * scores = reinterpret_cast<float *>(ws + l.scores_off);
    double * part = reinterpret_cast<double *>(ws + l.part_off);
    cudaError_t e = ensure_smem(k_fa_scores<G>, FA_SCORES_SMEM);
    if (e == cudaSuccess) e = ensure_smem(k_fa_pv<G>, fa_pv_smem<G>());
    if (e != cudaSuccess) return e;
    dim3 grid((unsigned)f.Hkv, (unsigned)f.T, (unsigned)f.S);
    e = alb_launch(k_fa_scores<G>, grid, dim3(128), FA_SCORES_SMEM, st, f.pdl, f.q, f.kc, f.Hq, f.Hkv, f.T,
                               f.pos0, f.pos_dev, f.scale, f.S, f.ncap, scores, smax);
    if (e != cudaSuccess) return e;
    e = alb_launch(k_fa_pv<G>, grid, dim3(128), fa_pv_smem<G>(), st, f.pdl, f.vc, f.Hq, f.Hkv, f.T, f.pos0,
                   f.pos_dev, f.S, f.ncap, (const float *)scores, (const float *)smax, part, f.out);
    if (e != cudaSuccess || f.S == 1) return e;
    return alb_launch(k_fa_merge<G>, dim3((unsigned)f.Hq, (unsigned)f.T), dim3(1024), 0, st, f.pdl,
                      (const double *)part, f.Hq, f.T, f.S, f.pos0, f.pos_dev, f.out, static_cast<uint8_t *>(f.xq));
}

// The split path's merge writes f.xq itself; the one-CTA paths quantize out after.
template <int G>
static cudaError_t launch_fa_t(const FlashArgs & f, cudaStream_t st) {
    const cudaError_t e = launch_fa_core<G>(f, st);
    if (e != cudaSuccess || !f.xq || f.S > 1) return e;
    return launch_quantize_q8_0(f.out, f.xq, (int64_t)f.T * f.Hq * 128, f.pdl, st);
}

cudaError_t launch_flash_attn(const FlashArgs & f, cudaStream_t st) {
    if (f.ncap <= 0 || f.Hkv <= 0 || f.Hq % f.Hkv != 0) return cudaErrorInvalidValue;
    switch (f.Hq / f.Hkv) {
        case 1: return launch_fa_t<1>(f, st);
        case 2: return launch_fa_t<2>(f, st);
        case 4: return launch_fa_t<4>(f, st);
        case 8: return launch_fa_t<8>(f, st);
        default: return cudaErrorInvalidValue;
    }
}

// ------------------------------------------------------------------- argmax
// sample_none / std::max_element (sampler.cpp:34-36): first index of the max.
// Each CTA reduces a contiguous chunk to (value, index); the last CTA (atomic
// ticket) reduces the candidates.  Keys order by value then by LOWER index.
__device__ __forceinline__ unsigned long long am_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);       // order-preserving
    return ((unsigned long long)u << 32) | (uint32_t)(0x7FFFFFFF - idx);
}

__global__ void __launch_bounds__(512)
k_argmax(const float * __restrict__ x, int64_t n, int64_t idx_base, unsigned long long * __restrict__ cand,
         int * __restrict__ ticket, unsigned long long * __restrict__ key_out, int32_t * __restrict__ idx_out) {
    __shared__ unsigned long long red[16];
    __shared__ int last;
    alb_pdl_wait();
    const int64_t chunk = (n + gridDim.x - 1) / gridDim.x;
    const int64_t b0 = (int64_t)blockIdx.x * chunk, b1 = min(n, b0 + chunk);
    unsigned long long best = 0;
    for (int64_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) {
        const unsigned long long k = am_key(x[i], (int)(i + idx_base));
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
        cand[blockIdx.x] = best;
        __threadfence();
        last = (atomicAdd(ticket, 1) == (int)gridDim.x - 1);
    }
    __syncthreads();
    if (!last) { alb_pdl_trigger(); return; }
    __threadfence();
    if (threadIdx.x == 0) {
        unsigned long long b = 0;
        for (unsigned i = 0; i < gridDim.x; ++i) { const unsigned long long k = __ldcg(cand + i); b = k > b ? k : b; }
        if (key_out) *key_out = b;
        if (idx_out) *idx_out = 0x7FFFFFFF - (int32_t)(b & 0xFFFFFFFFu);
        *ticket = 0;
    }
    alb_pdl_trigger();
}

__global__ void k_key_to_index(const unsigned long long * __restrict__ key, int32_t * __restrict__ idx) {
    alb_pdl_wait();
    *idx = 0x7FFFFFFF - (int32_t)(*key & 0xFFFFFFFFu);
    alb_pdl_trigger();
}

cudaError_t launch_argmax(const float * x, int64_t n, int64_t idx_base, void * scratch,
                          unsigned long long * key_out, int32_t * idx_out, bool pdl, cudaStream_t st) {
    const int grid = 64;
    unsigned long long * cand = reinterpret_cast<unsigned long long *>(scratch);
    int * ticket = reinterpret_cast<int *>(cand + grid);
    return alb_launch(k_argmax, dim3(grid), dim3(512), 0, st, pdl, x, n, idx_base, cand, ticket, key_out, idx_out);
}

cudaError_t launch_key_to_index(const unsigned long long * key, int32_t * idx, bool pdl, cudaStream_t st) {
    return alb_launch(k_key_to_index, dim3(1), dim3(1), 0, st, pdl, key, idx);
}

// --------------------------------------------------------- standalone ops
// rms_norm_f32 + MUL (ops.cpp:680-724, binary.cpp): one CTA per row.
__global__ void __launch_bounds__(256)
k_rms_norm(const float * __restrict__ x, const float * __restrict__ w, float * __restrict__ y, int64_t n, float eps) {
    const float * xr = x + (size_t)blockIdx.x * n;
    float * yr = y + (size_t)blockIdx.x * n;
    __shared__ double red[8];
    alb_pdl_wait();
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += 256) { const float v = xr[i]; s += (double)__fmul_rn(v, v); }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    const float mean = (float)(t / (double)n);
    const float scale = 1.0f / sqrtf(__fadd_rn(mean, eps));
    for (int64_t i = threadIdx.x; i < n; i += 256) {
        const float v = __fmul_rn(xr[i], scale);
        yr[i] = w ? __fmul_rn(v, w[i]) : v;
    }
    alb_pdl_trigger();
}

// swiglu_f32 (ops.cpp:1038-1092, arm.cpp:1789-1809): y = silu(g) * u
__global__ void k_swiglu(const float * __restrict__ g, const float * __restrict__ u, float * __restrict__ y, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    alb_pdl_wait();
    if (i < n) y[i] = alb_swiglu1(g[i], u[i]);
    alb_pdl_trigger();
}

// RMSNorm (+ MUL by w) then quantize_row_q8_0 of the result (arm.cpp:1819-1853):
// CTA (row, j) forms the row's sum of squares (every CTA of the row in the same
// order) and warp w quantizes block 8j + w of the normalized row (lane =
// element), so the Q8_0 records are those of the fp32 values y.
__global__ void __launch_bounds__(256)
k_rms_norm_q8(const float * __restrict__ x, const float * __restrict__ w, float * __restrict__ y,
              uint8_t * __restrict__ yq, int64_t n, float eps) {
    const float * xr = x + (size_t)blockIdx.x * n;
    __shared__ double red[8];
    alb_pdl_wait();
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += 256) { const float v = xr[i]; s += (double)__fmul_rn(v, v); }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    const float mean = (float)(t / (double)n);
    const float scale = 1.0f / sqrtf(__fadd_rn(mean, eps));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t nb = n / 32;
    uint8_t * qr = yq + (size_t)blockIdx.x * nb * 34;
    const int64_t b = (int64_t)blockIdx.y * 8 + warp;
    if (b < nb) {
        const int64_t i = b * 32 + lane;
        float v = __fmul_rn(xr[i], scale);
        if (w) v = __fmul_rn(v, w[i]);
        if (y) y[(size_t)blockIdx.x * n + i] = v;
        int8_t q; uint16_t dh;
        q8_block_lane(v, q, dh);
        if (lane == 0) *reinterpret_cast<uint16_t *>(qr + b * 34) = dh;
        qr[b * 34 + 2 + lane] = (uint8_t)q;
    }
    alb_pdl_trigger();
}

// swiglu (ops.cpp:1038-1092) then quantize_row_q8_0 of the product: one warp per block.
__global__ void __launch_bounds__(256)
k_swiglu_q8(const float * __restrict__ g, const float * __restrict__ u, float * __restrict__ y,
            uint8_t * __restrict__ yq, int64_t n_blocks) {
    const int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    alb_pdl_wait();
    if (b < n_blocks) {
        const int64_t i = b * 32 + lane;
        const float v = alb_swiglu1(g[i], u[i]);
        if (y) y[i] = v;
        int8_t q; uint16_t dh;
        q8_block_lane(v, q, dh);
        if (lane == 0) *reinterpret_cast<uint16_t *>(yq + b * 34) = dh;
        yq[b * 34 + 2 + lane] = (uint8_t)q;
    }
    alb_pdl_trigger();
}

cudaError_t launch_rms_norm_q8(const float * x, const float * w, float * y, void * yq, int64_t rows, int64_t n,
                               float eps, bool pdl, cudaStream_t st) {
    return alb_launch(k_rms_norm_q8, dim3((unsigned)rows, (unsigned)((n / 32 + 7) / 8)), dim3(256), 0, st, pdl, x,
                      w, y, static_cast<uint8_t *>(yq), n, eps);
}

cudaError_t launch_swiglu_q8(const float * g, const float * u, float * y, void * yq, int64_t n, bool pdl,
                             cudaStream_t st) {
    const int64_t nb = n / 32;
    return alb_launch(k_swiglu_q8, dim3((unsigned)((nb + 7) / 8)), dim3(256), 0, st, pdl, g, u, y,
                      static_cast<uint8_t *>(yq), nb);
}

cudaError_t launch_embed(const uint8_t * W, int64_t vocab, int64_t E, const int32_t * tokens, int T, float * x,
                         unsigned long long * key_reset, bool pdl, cudaStream_t st) {
    const int64_t n = (int64_t)T * (E / 32);
    return alb_launch(k_embed_q4_0, dim3((unsigned)((n + 127) / 128)), dim3(128), 0, st, pdl, W, tokens, T, E, vocab,
                      x, device_error_ptr(), key_reset);
}

cudaError_t launch_qk_norm_rope_kv(const QkvArgs & a, cudaStream_t st) {
    dim3 grid((unsigned)(a.Hq + 2 * a.Hkv), (unsigned)a.T);
    return alb_launch(k_qk_norm_rope_kv, grid, dim3(128), 0, st, a.pdl, a.qkv, a.qkv_stride, a.Hq, a.Hkv,
                      a.q_norm, a.k_norm, a.eps, a.rope, a.pos0, a.pos_dev, a.q_out, a.kc, a.vc,
                      (int64_t)a.Hkv * 128);
}

cudaError_t launch_rms_norm(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps, bool pdl,
                            cudaStream_t st) {
    return alb_launch(k_rms_norm, dim3((unsigned)rows), dim3(256), 0, st, pdl, x, w, y, n, eps);
}

cudaError_t launch_swiglu(const float * g, const float * u, float * y, int64_t n, bool pdl, cudaStream_t st) {
    return alb_launch(k_swiglu, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, pdl, g, u, y, n);
}

}  // namespace alb
