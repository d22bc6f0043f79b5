/*
 * ArcLight decode/prefill hot-path ORACLE -- test infrastructure only.
 *
 * This is a plain-C, CPU restatement of the reference's nnml arithmetic on the
 * Qwen3 Q4_0 decode/prefill path (OpenBMB/ArcLight, `nnml/src/ops/...`).  It is
 * the CHECKER for the CUDA product in `arclight_b200/`: only `tests/`,
 * `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference` legs of
 * `bench.py` may load it.  The product never links, calls or falls back to it.
 *
 * Every function cites the reference file:line whose semantics it restates.
 * The reference's own portable sources are additionally compiled (shimmed) into
 * `oracle/_ref/` by `oracle/Makefile`; `tests/golden/make_golden.py` runs both and
 * commits the reference outputs as fixtures, which pin this restatement.  The
 * NEON-only functions of `nnml/src/ops/arm/{arm,gemm}.cpp` cannot be compiled on
 * x86; they are restated here from their source (parity of those is pinned by
 * the KATs derived from the reference code, see tests/test_oracle_golden.py).
 */
#ifndef ARCLIGHT_ORACLE_H
#define ARCLIGHT_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK 32
/* block_q4_0: nnml.h:646-651 (fp16 d + 16 nibble bytes = 18 B) */
typedef struct { uint16_t d; uint8_t qs[16]; } orc_block_q4_0;
/* block_q8_0: nnml.h:695-700 (fp16 d + 32 int8 = 34 B) */
typedef struct { uint16_t d; int8_t qs[32]; } orc_block_q8_0;
/* block_q4_0x4 (ops.h:225-233, block<4,4>): 4 fp16 d + 64 interleaved bytes */
typedef struct { uint16_t d[4]; uint8_t qs[64]; } orc_block_q4_0x4;

/* ---- fp16 <-> fp32 (ops.h:276-324, RNE) ---- */
uint16_t orc_fp32_to_fp16(float f);
float    orc_fp16_to_fp32(uint16_t h);

/* ---- synthetic-input generator (not reference code: defines the seeded data) ---- */
uint64_t orc_splitmix64(uint64_t x);
void     orc_normal_table(float * table /* [65537] */);
float    orc_normal(const float * table, uint64_t seed, uint64_t idx);
uint64_t orc_tensor_seed(uint64_t model_seed, int layer, int kind);

/* ---- quantizers ---- */
void orc_quantize_row_q4_0(const float * x, orc_block_q4_0 * y, int64_t k);     /* types.cpp:352-378 */
void orc_dequantize_row_q4_0(const orc_block_q4_0 * x, float * y, int64_t k);   /* types.cpp:337-350 */
void orc_quantize_row_q8_0(const float * x, orc_block_q8_0 * y, int64_t k);     /* arm.cpp:1819-1853 (RNE) */
void orc_quantize_row_q8_0_ref(const float * x, orc_block_q8_0 * y, int64_t k); /* types.cpp:494-514 (roundf) */
void orc_dequantize_row_q8_0(const orc_block_q8_0 * x, float * y, int64_t k);   /* types.cpp:483-492 */
/* make_block_q4_0x4 / repack_q4_0_to_q4_0_4_bl (types.cpp:133-197), interleave 4 */
int  orc_repack_q4_0_4x4(const orc_block_q4_0 * src, orc_block_q4_0x4 * dst, int64_t nrow, int64_t k);

/* ---- mat-vec ---- */
/* nnml_gemv_q4_0_4x4_q8_0 NEON path (gemm.cpp:127-190): per row n,
 *   I(n,b) = sum_j (lo_j-8) a_j + (hi_j-8) a_{j+16}  (int32, exact)
 *   y[n]   = fma chain over b of float(I) * (f32(dx_b) * f32(dw_b)).
 * W is in the reference's un-repacked block_q4_0 row layout [N][K/32]
 * (the 4x4 interleave only reorders bytes).  block_dots (nullable) [N][K/32]. */
void orc_gemv_q4_0_q8_0(const orc_block_q4_0 * W, const orc_block_q8_0 * xq, float * y,
                        int64_t N, int64_t K, int32_t * block_dots, int n_threads);
/* Exactly rounded twin: block terms summed exactly in double, rounded once
 * (order independent; within a few fp32 ulps of the NEON chain). */
void orc_gemv_q4_0_q8_0_exact(const orc_block_q4_0 * W, const orc_block_q8_0 * xq, float * y,
                              int64_t N, int64_t K, int n_threads);
/* Tensor-parallel twin for column-split matrices (O, down; model.cpp:21-54): node
 * j's exactly rounded partial over its K/tp column slice, partials added in node
 * order in fp32 (GATHER, ops.cpp:1465-1511). */
void orc_gemv_q4_0_q8_0_exact_tp(const orc_block_q4_0 * W, const orc_block_q8_0 * xq, float * y,
                                 int64_t N, int64_t K, int tp, int n_threads);
/* Tensor-parallel NEON chain (the reference's TP arithmetic for O / down): node
 * j's partial is the fp32 chain over its K/tp column slice, partials added in
 * node order in fp32 (GATHER, ops.cpp:1465-1511). */
void orc_gemv_q4_0_q8_0_tp(const orc_block_q4_0 * W, const orc_block_q8_0 * xq, float * y,
                           int64_t N, int64_t K, int tp, int n_threads);
/* nnml_vec_dot_q4_0_q8_0 NEON path (arm.cpp:633-692): generic mul_mat (lm_head). */
float orc_vec_dot_q4_0_q8_0(const orc_block_q4_0 * x, const orc_block_q8_0 * y, int64_t k);
void  orc_mul_mat_generic(const orc_block_q4_0 * W, const orc_block_q8_0 * xq, float * y,
                          int64_t N, int64_t K, int n_threads);

/* ---- elementwise ---- */
/* rms_norm_f32 (ops.cpp:680-724) then MUL by w (binary.cpp:15-23; w nullable) */
void orc_rms_norm(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps);
/* rope NEOX, ext_factor 0, freq_scale 1, attn_factor 1 (ops.cpp:747-961) */
void orc_rope_cache(int32_t pos, int64_t n_dims, float theta_scale, float * cache /* [n_dims] cos,sin */);
void orc_rope_neox(const float * x, float * y, int64_t n_heads, int64_t head_dim, int32_t pos, float freq_base);
/* nnml_v_expf restated per lane (arm.cpp:1757-1787) */
float orc_neon_expf(float x);
/* swiglu: silu(g)*u (ops.cpp:1038-1092, arm.cpp:1789-1809) */
void orc_swiglu(const float * g, const float * u, float * y, int64_t n);
/* GATHER sum (ops.cpp:1465-1511, arm.cpp:2435-2451): dst = src0 + src1 + ... */
void orc_gather_sum(const float * const * srcs, int n_srcs, float * dst, int64_t n);

/* ---- flash attention (arm.cpp:2196-2433) ----
 * q    : [T][n_head][D] fp32
 * k,v  : [n_cells][n_head_kv][D] fp16 (cell-major, the reference's FA-mode K/V views,
 *        cgraph.cpp:1057-1112 with v_trans=false)
 * kv_len[t]: token t attends cells [0, kv_len[t]) (the causal mask of
 *        cgraph.cpp:1224-1261 for one sequence filled in order)
 * out  : [T][n_head][D] fp32
 * mode 0: fp32 scores, global-max softmax with nnml_v_expf, double sums in a
 *         canonical order: cells in order within chunks of ORC_FA_CHUNK cells,
 *         chunk sums added in chunk order (the semantics of the CUDA kernels,
 *         independent of how they split the cells);
 * mode 1: ARM-faithful fp16 VKQ/KQ accumulation with online softmax;
 * mode 2: the same function in fp64 (scores, exp, sums), rounded once: the
 *         yardstick that modes 0 and 1 are measured against. */
#define ORC_FA_CHUNK 128
/* at most this many superchunks: a superchunk is ceil(chunks / ORC_FA_SUPER)
 * consecutive chunks (one chunk up to 64 chunks = 8192 cells) */
#define ORC_FA_SUPER 64
void orc_flash_attn(const float * q, const uint16_t * k, const uint16_t * v, const int32_t * kv_len,
                    int64_t T, int64_t n_head, int64_t n_head_kv, int64_t D, float scale,
                    int mode, float * out);
/* the same over n_threads threads (the (token, head) outputs split among them;
 * results identical to orc_flash_attn) */
void orc_flash_attn_mt(const float * q, const uint16_t * k, const uint16_t * v, const int32_t * kv_len,
                       int64_t T, int64_t n_head, int64_t n_head_kv, int64_t D, float scale,
                       int mode, float * out, int n_threads);

/* ---- Qwen3 model (qwen3.cpp:174-275), synthetic seeded weights ---- */
typedef struct {
    int32_t n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff, n_vocab, tied;
    float   eps, freq_base;
} orc_qwen3_config;

enum {
    ORC_T_TOK_EMBD = 0, ORC_T_OUTPUT = 1, ORC_T_OUTPUT_NORM = 2,
    ORC_T_ATTN_NORM = 3, ORC_T_WQ = 4, ORC_T_WK = 5, ORC_T_WV = 6, ORC_T_WO = 7,
    ORC_T_Q_NORM = 8, ORC_T_K_NORM = 9, ORC_T_FFN_NORM = 10,
    ORC_T_GATE = 11, ORC_T_UP = 12, ORC_T_DOWN = 13,
};

typedef struct orc_model orc_model;
orc_model * orc_model_create(const orc_qwen3_config * cfg, uint64_t seed, int32_t max_ctx, int n_threads);
void        orc_model_free(orc_model * m);
/* raw weight access (for checking the product's generator) */
const orc_block_q4_0 * orc_model_q4_tensor(orc_model * m, int layer, int kind, int64_t * rows, int64_t * cols);
const float *          orc_model_f32_tensor(orc_model * m, int layer, int kind, int64_t * n);
/* One ubatch of T tokens at positions [pos0, pos0+T).  fa_mode as orc_flash_attn.
 * logits: [n_vocab] of the LAST token (qwen3.cpp:235-238 keeps only the last row).
 * hidden (nullable): final-normed hidden state of the last token [n_embd]. */
int  orc_model_forward(orc_model * m, const int32_t * tokens, int32_t T, int32_t pos0,
                       int fa_mode, float * logits, float * hidden);
void orc_model_reset(orc_model * m);
/* Long-context benchmark pre-fill: K and V of positions [0, n_pos) of every
 * layer set to fp16(N(0,1)) from the seeded generator, element (cell, e) of
 * layer l drawn at index cell * Dkv + e under orc_tensor_seed(seed, l, 62 | 63). */
void orc_model_fill_kv(orc_model * m, int32_t n_pos, uint64_t seed);
/* exact == 0 (default): the reference's NEON fp32 chains (gemv for the
 * projections, nnml_vec_dot_q4_0_q8_0 lanes for the lm head); != 0: every
 * mat-vec exactly rounded (orc_gemv_q4_0_q8_0_exact, for error studies). */
void orc_model_set_exact(orc_model * m, int exact);
/* tp > 1: the O and down projections as tp node partials added in node order,
 * then the residual (qwen3.cpp:232-241,262-270 with is_tp). */
void orc_model_set_tp(orc_model * m, int tp);
/* greedy argmax (sampler.cpp:34-36: std::max_element => first maximum) */
int32_t orc_argmax(const float * x, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
