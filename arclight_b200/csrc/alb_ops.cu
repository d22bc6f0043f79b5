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
// SET_ROWS to fp16 (ops.cpp:135-181, as cpy_k / cpy_v use it with the KV cache's
// cell indices, cgraph.cpp:1114-1180): dst[idx[r]] = fp16(src[r]) with RNE
// (common.cpp:19-24).  One thread per 8 values (one 16-byte store); a row whose
// index lies outside [0, dst_rows) is skipped and sets the device error word.
__global__ void k_set_rows_f16(const float * __restrict__ src, int64_t n_rows, int64_t row_len,
                               const int64_t * __restrict__ idx, uint16_t * __restrict__ dst, int64_t dst_rows,
                               int * err) {
    const int64_t per_row = row_len / 8;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows * per_row) return;
    const int64_t r = i / per_row, c = (i - r * per_row) * 8;
    const int64_t d = idx[r];
    if (d < 0 || d >= dst_rows) {
        if (c == 0) atomicExch(err, ALB_DEVERR_BAD_INDEX);
        return;
    }
    const float4 a = *reinterpret_cast<const float4 *>(src + r * row_len + c);
    const float4 b = *reinterpret_cast<const float4 *>(src + r * row_len + c + 4);
    uint4 o;
    o.x = (uint32_t)alb_f2h(a.x) | ((uint32_t)alb_f2h(a.y) << 16);
    o.y = (uint32_t)alb_f2h(a.z) | ((uint32_t)alb_f2h(a.w) << 16);
    o.z = (uint32_t)alb_f2h(b.x) | ((uint32_t)alb_f2h(b.y) << 16);
    o.w = (uint32_t)alb_f2h(b.z) | ((uint32_t)alb_f2h(b.w) << 16);
    *reinterpret_cast<uint4 *>(dst + d * row_len + c) = o;
}

// GET_ROWS of fp16 rows (ops.cpp:12-131 for an F16 table): dst[r] = src[idx[r]],
// one thread per 8 values; a row whose index lies outside [0, src_rows) is
// written as zeros and sets the device error word.
__global__ void k_get_rows_f16(const uint16_t * __restrict__ src, int64_t src_rows, int64_t row_len,
                               const int64_t * __restrict__ idx, int64_t n_rows, uint16_t * __restrict__ dst,
                               int * err) {
    const int64_t per_row = row_len / 8;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows * per_row) return;
    const int64_t r = i / per_row, c = (i - r * per_row) * 8;
    const int64_t s = idx[r];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (s >= 0 && s < src_rows) {
        v = *reinterpret_cast<const uint4 *>(src + s * row_len + c);
    } else if (c == 0) {
        atomicExch(err, ALB_DEVERR_BAD_INDEX);
    }
    *reinterpret_cast<uint4 *>(dst + r * row_len + c) = v;
}

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
// (set_rows, ops.cpp:135-181); V heads are stored as is.  With pos_tok /
// cell_tok (device, per token) token t takes position pos_tok[t] and stores
// into cell cell_tok[t] instead (a ubatch of several sequences placed by the
// KV-cache manager); a position outside the RoPE table or a cell outside the
// cache skips the token and sets the device error word.
// Block = 128 threads (one per dimension), grid = (Hq + 2*Hkv, T).
__global__ void __launch_bounds__(128)
k_qk_norm_rope_kv(const float * __restrict__ qkv, int64_t qkv_stride, int Hq, int Hkv,
                  const float * __restrict__ qn_w, const float * __restrict__ kn_w, float eps,
                  const float2 * __restrict__ rope, int32_t pos0, const int32_t * __restrict__ pos_dev,
                  float * __restrict__ q_out, uint16_t * __restrict__ kc, uint16_t * __restrict__ vc,
                  int64_t kv_row, const int32_t * __restrict__ pos_tok, const int64_t * __restrict__ cell_tok,
                  int64_t n_cells, int32_t max_pos, int * err) {
    const int head = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
    const int lane = d & 31, warp = d >> 5;
    alb_pdl_wait();
    const int32_t pos = pos_tok ? pos_tok[t] : (pos_dev ? pos_dev[0] : pos0) + t;
    const int64_t cell = cell_tok ? cell_tok[t] : (int64_t)pos;
    if ((pos_tok || cell_tok) && (pos < 0 || pos >= max_pos || cell < 0 || cell >= n_cells)) {
        if (d == 0) atomicExch(err, ALB_DEVERR_BAD_INDEX);   // the whole block leaves: no store, no read
        alb_pdl_trigger();
        return;
    }
    const float * src = qkv + (size_t)t * qkv_stride;
    __shared__ float buf[128];
    __shared__ double red[4];
    if (head >= Hq + Hkv) {   // V head: plain fp16 store
        const int hv = head - Hq - Hkv;
        vc[(size_t)cell * kv_row + hv * 128 + d] = alb_f2h(src[(Hq + Hkv) * 128 + hv * 128 + d]);
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
    buf[d] = v;
    __syncthreads();
    double tot = ((red[0] + red[1]) + red[2]) + red[3];
    __shared__ double seq_tot;
    if (!alb_rms_mean_certain(tot, 128)) {   // the reference's sequential sum (uniform branch)
        if (d == 0) seq_tot = alb_rms_seq_sum(buf, 128);
        __syncthreads();
        tot = seq_tot;
    }
    __syncthreads();   // buf is rewritten below
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
    else      kc[(size_t)cell * kv_row + hh * 128 + d] = alb_f2h(outv);
    alb_pdl_trigger();
}

// ------------------------------------------------------------ flash attention
// Prefill attention (T > 1 tokens, one split).  Semantics of the split-K
// kernels (alb_attn.cu, the oracle's mode 0): fp16-rounded Q, fp32 score
// chains, global-max softmax with the reference's NEON exp, sums of p and p * v
// in the canonical order -- cells in order in fp32 within 128-cell chunks, the
// chunk sums added in double in chunk order.
__device__ __forceinline__ void fa_cp16(void * dst, const void * src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(alb_smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void fa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void fa_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Prefill attention (ubatches of T > 1 tokens): one CTA per (KV head h, tile of
// TQ = 64/G tokens) computes the 64 rows (row r: token t0 + r/G, query head
// h*G + r%G) over K/V stages of 64 cells brought by cp.async (double-buffered),
// so each staged cell serves 64 rows instead of one.  Same arithmetic as the
// decode kernels: every score is the sequential fp32 fma chain over d of the
// fp16-rounded q (16 chains per thread: one cell, 16 rows); pass 1 takes the
// row maxima over each row's causal cells, pass 2 recomputes the same scores,
// forms p = v_expf(s - M) and accumulates the chunk's L (row threads) and
// O = fmaf(p, v, O) in fp32 as a register tile of 4 rows x 8 dims per thread,
// cell by cell in order; chunk sums join double superchunk and total sums.
static constexpr int FP_R = 64;                 // rows per CTA
static constexpr int FP_CH = 64;                // cells per stage (two stages per 128-cell chunk)
static constexpr int FP_KPITCH = 272;           // padded K row in shared memory
static constexpr int FP_PP = FP_CH + 4;         // padded row of p (floats): the row scans and the P.V
                                                // tile's rows r, r + 4 fall in distinct banks
static constexpr size_t FP_SMEM = (size_t)128 * FP_R * 4 + 2 * FP_CH * FP_KPITCH + 2 * FP_CH * 256 +
                                  (size_t)FP_R * FP_CH * 8 + (size_t)FP_R * 128 * 8;
                                  // q^T, K x2, V x2, p, O totals: 198,656 B

// The 16 score chains of two cells (K rows kr0, kr1 in shared memory) against
// rows 8*rg .. 8*rg+7 of q^T [128][FP_R]: a[8u + k] = cell u, row 8*rg + k, each
// the sequential fp32 fma chain over d.  Every broadcast q load feeds two
// cells' fmas (half the shared-memory loads per fma of one cell x 16 rows).
__device__ __forceinline__ void fp_scores2x8(const uint8_t * __restrict__ kr0, const uint8_t * __restrict__ kr1,
                                             const float * __restrict__ qT, int rg, float (&a)[16]) {
#pragma unroll
    for (int k = 0; k < 16; ++k) a[k] = 0.0f;
#pragma unroll 2
    for (int j = 0; j < 16; ++j) {
        const uint4 kv0 = *reinterpret_cast<const uint4 *>(kr0 + j * 16);
        const uint4 kv1 = *reinterpret_cast<const uint4 *>(kr1 + j * 16);
        const uint32_t w0[4] = {kv0.x, kv0.y, kv0.z, kv0.w}, w1[4] = {kv1.x, kv1.y, kv1.z, kv1.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&w0[e]));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&w1[e]));
#pragma unroll
            for (int hlf = 0; hlf < 2; ++hlf) {
                const float k0 = hlf ? f0.y : f0.x, k1 = hlf ? f1.y : f1.x;
                const float * qd = qT + (8 * j + 2 * e + hlf) * FP_R + 8 * rg;
                const float4 qa = *reinterpret_cast<const float4 *>(qd);
                const float4 qb = *reinterpret_cast<const float4 *>(qd + 4);
                const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    a[k] = __fmaf_rn(k0, qv[k], a[k]);
                    a[8 + k] = __fmaf_rn(k1, qv[k], a[8 + k]);
                }
            }
        }
    }
}

// STORE: pass 1 also writes every scaled score of the tile (64 rows x n cells)
// to the workspace `sws` (row stride `sstride`), and pass 2 reads them back --
// each thread re-reads exactly the values it wrote -- instead of recomputing
// the 128-long chains (bit-identical scores, no K stages in pass 2).
template <int G, bool STORE>
__global__ void __launch_bounds__(256, 1)
k_fa_prefill(const float * __restrict__ q, const uint16_t * __restrict__ kc, const uint16_t * __restrict__ vc, int Hq,
             int Hkv, int T, int32_t pos0, const int32_t * __restrict__ pos_dev, float scale, float * __restrict__ out,
             float * __restrict__ sws, int64_t sstride) {
    constexpr int TQ = FP_R / G;
    extern __shared__ __align__(16) uint8_t fp_sm[];
    float * qT = reinterpret_cast<float *>(fp_sm);                            // [128][FP_R]
    uint8_t * kst = fp_sm + (size_t)128 * FP_R * 4;                           // 2 x [FP_CH][FP_KPITCH]
    uint8_t * vst = kst + 2 * FP_CH * FP_KPITCH;                              // 2 x [FP_CH][256]
    float * pf = reinterpret_cast<float *>(vst + 2 * FP_CH * 256);            // [FP_R][FP_PP] p of the stage
    double * Otot = reinterpret_cast<double *>(pf + 2 * FP_R * FP_CH);         // [FP_R][128]
    __shared__ float Mrow[FP_R];
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
    // this tile's scores in the workspace: [FP_R rows][sstride cells]
    float * sreg = STORE ? sws + ((size_t)blockIdx.x * gridDim.y + blockIdx.y) * FP_R * (size_t)sstride : nullptr;
    auto issue = [&](int i, bool with_k, bool with_v) {
        if (i < nst) {
            const int cb = i * FP_CH, rows = min(FP_CH, n - cb);
            uint8_t * kd = kst + (i & 1) * FP_CH * FP_KPITCH;
            uint8_t * vd = vst + (i & 1) * FP_CH * 256;
            for (int p = tid; p < rows * 16; p += 256) {
                const int r = p >> 4, j = p & 15;
                const size_t src = (size_t)(cb + r) * row + (size_t)h * 128 + j * 8;
                if (with_k) fa_cp16(kd + r * FP_KPITCH + j * 16, kc + src);
                if (with_v) fa_cp16(vd + r * 256 + j * 16, vc + src);
            }
        }
        fa_commit();
    };
    // score phase: cells pr and pr + 32 of the stage, rows 8*rg .. 8*rg+7 (warp = row group)
    const int pr = tid & 31, rg = tid >> 5;
    // ---- pass 1: row maxima over the causal cells
    float mx[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) mx[k] = -INFINITY;
    issue(0, true, false);
    for (int i = 0; i < nst; ++i) {
        issue(i + 1, true, false);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();   // stage i (and q^T) visible
        const int cA = i * FP_CH + pr;
        if (cA < n) {   // (cell cA + 32 may lie past n: its chains are computed and dropped)
            float a[16];
            const uint8_t * ks = kst + (i & 1) * FP_CH * FP_KPITCH;
            fp_scores2x8(ks + pr * FP_KPITCH, ks + (pr + 32) * FP_KPITCH, qT, rg, a);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int c = cA + 32 * u;
                if (c < n) {
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int r = 8 * rg + k, tt = r / G;
                        const float v = __fmul_rn(a[8 * u + k], scale);
                        if (STORE) sreg[(size_t)r * sstride + c] = v;
                        if (tt < tn && c <= p0 + t0 + tt) mx[k] = fmaxf(mx[k], v);
                    }
                }
            }
        }
        __syncthreads();   // buffer i & 1 consumed before stage i + 2 refills it
    }
    fa_wait_all();
#pragma unroll
    for (int k = 0; k < 8; ++k) {   // warp rg holds every cell of rows 8*rg ..
        const float m = alb_warp_max(mx[k]);
        if (lane == 0) Mrow[8 * rg + k] = m;
    }
    // ---- pass 2: p, L and O (chunk partials: O in registers, L by row threads)
    const int r4 = (tid >> 4) * 4, d8 = (tid & 15) * 8;   // P.V tile of this thread
    float O[4][8];                                        // chunk sums (fp32, cells in order)
    double Osp[4][8];                                     // superchunk sums
    float Lc = 0.0f;                                      // thread r < FP_R: row r's chunk sum of p,
    double Lsp = 0.0, Lt = 0.0;                           // its superchunk and total sums
    // per row: its chunks (of its own causal cells) and chunks per superchunk
    // (the canonical order: chunk sums in order within superchunks of
    // ceil(chunks / 64) chunks, superchunk sums in order)
    int nch_u[4], scn_u[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int nr = p0 + t0 + (r4 + u) / G + 1;
        nch_u[u] = (nr + 127) / 128;
        scn_u[u] = nch_u[u] > 64 ? (nch_u[u] + 63) / 64 : 1;
    }
    const int nch_l = (p0 + t0 + (tid & (FP_R - 1)) / G + 1 + 127) / 128;
    const int scn_l = nch_l > 64 ? (nch_l + 63) / 64 : 1;
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int e = 0; e < 8; ++e) { O[u][e] = 0.0f; Osp[u][e] = 0.0; Otot[(r4 + u) * 128 + d8 + e] = 0.0; }
    issue(0, !STORE, true);
    for (int i = 0; i < nst; ++i) {
        issue(i + 1, !STORE, true);
        const int cA = i * FP_CH + pr;
        float a[16];   // scaled scores of cells cA, cA + 32 (STORE: read back, issued before the stage wait)
#pragma unroll
        for (int k = 0; k < 16; ++k) a[k] = 0.0f;
        if (STORE) {
#pragma unroll
            for (int u = 0; u < 2; ++u)
                if (cA + 32 * u < n)
#pragma unroll
                    for (int k = 0; k < 8; ++k) a[8 * u + k] = sreg[(size_t)(8 * rg + k) * sstride + cA + 32 * u];
        }
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();   // stage i visible; Mrow visible; pf free
        if (!STORE && cA < n) {
            const uint8_t * ks = kst + (i & 1) * FP_CH * FP_KPITCH;
            fp_scores2x8(ks + pr * FP_KPITCH, ks + (pr + 32) * FP_KPITCH, qT, rg, a);
#pragma unroll
            for (int k = 0; k < 16; ++k) a[k] = __fmul_rn(a[k], scale);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int c = cA + 32 * u;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int r = 8 * rg + k, tt = r / G;
                float v = 0.0f;
                if (c < n && tt < tn && c <= p0 + t0 + tt) v = alb_ref_expf(__fsub_rn(a[8 * u + k], Mrow[r]));
                pf[r * FP_PP + pr + 32 * u] = v;
            }
        }
        __syncthreads();
        if (tid < FP_R) {   // row tid's sum of p over the stage's cells, in order (masked cells add 0)
            const float * prow = pf + tid * FP_PP;
#pragma unroll 4
            for (int cc = 0; cc < FP_CH; cc += 4) {
                const float4 p4 = *reinterpret_cast<const float4 *>(prow + cc);
                Lc = __fadd_rn(Lc, p4.x);
                Lc = __fadd_rn(Lc, p4.y);
                Lc = __fadd_rn(Lc, p4.z);
                Lc = __fadd_rn(Lc, p4.w);
            }
        }
        const int rows = min(FP_CH, n - i * FP_CH);
        const uint8_t * vs = vst + (i & 1) * FP_CH * 256 + d8 * 2;
        // one cell of V (8 dims) into O's 4 rows, p from the given values
        auto pv_cell = [&](int cc, const float (&p)[4]) {
            const uint4 vv = *reinterpret_cast<const uint4 *>(vs + cc * 256);
            const uint32_t wd[4] = {vv.x, vv.y, vv.z, vv.w};
            float vf[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&wd[e]));
                vf[2 * e] = f.x;
                vf[2 * e + 1] = f.y;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int e = 0; e < 8; ++e) O[u][e] = __fmaf_rn(p[u], vf[e], O[u][e]);   // fp32, cells in order
        };
        int cc = 0;
        for (; cc + 4 <= rows; cc += 4) {   // p of 4 cells per row in one 16-byte load
            float4 p4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) p4[u] = *reinterpret_cast<const float4 *>(pf + (r4 + u) * FP_PP + cc);
            { const float p[4] = {p4[0].x, p4[1].x, p4[2].x, p4[3].x}; pv_cell(cc, p); }
            { const float p[4] = {p4[0].y, p4[1].y, p4[2].y, p4[3].y}; pv_cell(cc + 1, p); }
            { const float p[4] = {p4[0].z, p4[1].z, p4[2].z, p4[3].z}; pv_cell(cc + 2, p); }
            { const float p[4] = {p4[0].w, p4[1].w, p4[2].w, p4[3].w}; pv_cell(cc + 3, p); }
        }
        for (; cc < rows; ++cc) {   // the ragged tail of the last stage
            float p[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) p[u] = pf[(r4 + u) * FP_PP + cc];
            pv_cell(cc, p);
        }
        if ((i & 1) == 1 || i == nst - 1) {   // a 128-cell chunk ends: its sums join the superchunk's
            const int j = i >> 1;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const bool send = (j + 1) % scn_u[u] == 0 || j == nch_u[u] - 1;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    Osp[u][e] += (double)O[u][e];
                    O[u][e] = 0.0f;
                    if (send) { Otot[(r4 + u) * 128 + d8 + e] += Osp[u][e]; Osp[u][e] = 0.0; }
                }
            }
            if (tid < FP_R) {
                Lsp += (double)Lc;
                Lc = 0.0f;
                if ((j + 1) % scn_l == 0 || j == nch_l - 1) { Lt += Lsp; Lsp = 0.0; }
            }
        }
        __syncthreads();   // pf and buffer i & 1 consumed
    }
    fa_wait_all();
    __shared__ double Lrow[FP_R];
    if (tid < FP_R) Lrow[tid] = Lt;
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int r = r4 + u, tt = r / G, g = r % G;
        if (tt >= tn) continue;
        const double Ls = Lrow[r];
        float * o = out + ((size_t)(t0 + tt) * Hq + h * G + g) * 128 + d8;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = Ls > 0.0 ? __double2float_rn(Otot[r * 128 + d8 + e] / Ls) : 0.0f;
    }
    alb_pdl_trigger();
}

cudaError_t launch_set_rows_f16(const float * src, int64_t n_rows, int64_t row_len, const int64_t * idx, uint16_t * dst,
                                int64_t dst_rows, cudaStream_t st) {
    int * err = device_error_ptr();
    if (!err) return cudaErrorMemoryAllocation;
    const int64_t n = n_rows * (row_len / 8);
    k_set_rows_f16<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, n_rows, row_len, idx, dst, dst_rows, err);
    return cudaGetLastError();
}

cudaError_t launch_get_rows_f16(const uint16_t * src, int64_t src_rows, int64_t row_len, const int64_t * idx,
                                int64_t n_rows, uint16_t * dst, cudaStream_t st) {
    int * err = device_error_ptr();
    if (!err) return cudaErrorMemoryAllocation;
    const int64_t n = n_rows * (row_len / 8);
    k_get_rows_f16<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, src_rows, row_len, idx, n_rows, dst, err);
    return cudaGetLastError();
}

size_t flash_attn_ws_bytes(int Hq, int Hkv, int T, int S, int ncap) {
    return split_attn_ws_bytes(Hq, Hkv, T, S, ncap);
}

// Prefill ubatches (T > 1, one split) take the token-tiled kernel and need no
// workspace; every other call runs the split kernels on the workspace.
bool flash_attn_uses_ws(int Hq, int Hkv, int T, int S, int ncap) {
    (void)Hq; (void)Hkv; (void)ncap;
    return !(T > 1 && S == 1);
}

// Score workspace of the stored-score prefill path: FP_R rows x sstride cells
// per CTA (KV head x token tile), sstride = ncap rounded up to 4.
size_t fa_prefill_scores_bytes(int Hq, int Hkv, int T, int ncap) {
    if (Hkv <= 0 || Hq % Hkv != 0 || T <= 1) return 0;
    const int TQ = FP_R / (Hq / Hkv);
    return (size_t)Hkv * ((T + TQ - 1) / TQ) * FP_R * (size_t)((ncap + 3) & ~3) * 4;
}

template <int G, bool STORE>
static cudaError_t launch_fa_prefill_t(const FlashArgs & f, cudaStream_t st) {
    cudaError_t e = ensure_smem(k_fa_prefill<G, STORE>, FP_SMEM);
    if (e != cudaSuccess) return e;
    constexpr int TQ = FP_R / G;
    const dim3 grid((unsigned)f.Hkv, (unsigned)((f.T + TQ - 1) / TQ));
    return alb_launch(k_fa_prefill<G, STORE>, grid, dim3(256), FP_SMEM, st, f.pdl, f.q, f.kc, f.vc, f.Hq, f.Hkv, f.T,
                      f.pos0, f.pos_dev, f.scale, f.out, f.sws, (int64_t)((f.ncap + 3) & ~3));
}

template <int G>
static cudaError_t launch_fa_prefill(const FlashArgs & f, cudaStream_t st) {
    cudaError_t e = f.sws ? launch_fa_prefill_t<G, true>(f, st) : launch_fa_prefill_t<G, false>(f, st);
    if (e != cudaSuccess || !f.xq) return e;
    return launch_quantize_q8_0(f.out, f.xq, (int64_t)f.T * f.Hq * 128, f.pdl, st);
}

cudaError_t launch_flash_attn(const FlashArgs & f, cudaStream_t st) {
    if (f.ncap <= 0 || f.Hkv <= 0 || f.Hq % f.Hkv != 0) return cudaErrorInvalidValue;
    if (f.T > 1 && f.S == 1) {
        switch (f.Hq / f.Hkv) {
            case 1: return launch_fa_prefill<1>(f, st);
            case 2: return launch_fa_prefill<2>(f, st);
            case 4: return launch_fa_prefill<4>(f, st);
            case 8: return launch_fa_prefill<8>(f, st);
            default: return cudaErrorInvalidValue;
        }
    }
    return launch_split_attn(f, st);
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
    const double inv_n = 1.0 / (double)n;
    alb_pdl_wait();
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += 256) { const float v = xr[i]; s += (double)__fmul_rn(v, v); }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    const double t = alb_tree_sum<8>(red);
    float mean;
    if (!alb_rms_mean_cert(t, (int)n, inv_n, mean)) {   // the reference's sequential sum (uniform branch)
        __syncthreads();
        if (threadIdx.x == 0) red[0] = alb_rms_seq_sum(xr, (int)n);
        __syncthreads();
        mean = (float)(red[0] / (double)n);
    }
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
    const double inv_n = 1.0 / (double)n;
    alb_pdl_wait();
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += 256) { const float v = xr[i]; s += (double)__fmul_rn(v, v); }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    const double t = alb_tree_sum<8>(red);
    float mean;
    if (!alb_rms_mean_cert(t, (int)n, inv_n, mean)) {   // the reference's sequential sum (uniform branch)
        __syncthreads();
        if (threadIdx.x == 0) red[0] = alb_rms_seq_sum(xr, (int)n);
        __syncthreads();
        mean = (float)(red[0] / (double)n);
    }
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
    int * err = nullptr;
    if (a.pos_tok || a.cell_tok) {
        err = device_error_ptr();
        if (!err) return cudaErrorMemoryAllocation;
    }
    return alb_launch(k_qk_norm_rope_kv, grid, dim3(128), 0, st, a.pdl, a.qkv, a.qkv_stride, a.Hq, a.Hkv,
                      a.q_norm, a.k_norm, a.eps, a.rope, a.pos0, a.pos_dev, a.q_out, a.kc, a.vc,
                      (int64_t)a.Hkv * 128, a.pos_tok, a.cell_tok, a.n_cells, a.max_pos, err);
}

cudaError_t launch_rms_norm(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps, bool pdl,
                            cudaStream_t st) {
    return alb_launch(k_rms_norm, dim3((unsigned)rows), dim3(256), 0, st, pdl, x, w, y, n, eps);
}

cudaError_t launch_swiglu(const float * g, const float * u, float * y, int64_t n, bool pdl, cudaStream_t st) {
    return alb_launch(k_swiglu, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, pdl, g, u, y, n);
}

}  // namespace alb
