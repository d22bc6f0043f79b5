/*
 * alb_cuda.h -- C ABI of the ArcLight B200 hot path (libalb_cuda.so).
 *
 * Drop-in boundary for the nnml operators of OpenBMB/ArcLight's Qwen3 Q4_0
 * decode/prefill path.  Every entry point takes caller-owned device pointers,
 * plain sizes and a cudaStream_t (passed as void *), is stream ordered, never
 * allocates on the hot path and returns an int status (ALB_OK = 0, < 0 error;
 * alb_last_error() gives the message).  The reference's ops return void and
 * abort (nnml.h:97-111); callers that want that behaviour abort on status < 0.
 *
 * Each declaration cites the reference interface it replaces (file:line in the
 * ArcLight tree).  Layouts:
 *   block_q4_0  : {fp16 d; uint8 qs[16]}  18 B per 32 values (nnml.h:646-651)
 *   block_q8_0  : {fp16 d; int8  qs[32]}  34 B per 32 values (nnml.h:695-700)
 *   alb Q4_0 GPU layout (what alb_repack_q4_0 writes; replaces block_q4_0x4),
 *       row-interleaved: row n occupies alb_q4_0_row_bytes(K) bytes at
 *       n * alb_q4_0_row_bytes(K): the 16 qs bytes of each of its K/32 blocks
 *       (block b at 16*b, block_q4_0.qs unchanged), then the K/32 fp16 scales
 *       padded with zeros to a multiple of 8 entries (16 bytes).  A run of
 *       consecutive rows is one contiguous 16-byte aligned range.
 *   activations fp32 row-major; KV cache fp16 [cells][n_head_kv][head_dim].
 */
#ifndef ALB_CUDA_H
#define ALB_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ALB_API __attribute__((visibility("default")))
#else
#define ALB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ALB_OK = 0,
    ALB_ERR_INVALID = -1,     /* bad argument (null pointer, unsupported shape) */
    ALB_ERR_CUDA = -2,        /* CUDA runtime error (message in alb_last_error) */
    ALB_ERR_NCCL = -3,        /* collective error or abort */
    ALB_ERR_TIMEOUT = -4,     /* a bounded device/host wait expired */
    ALB_ERR_UNSUPPORTED = -5, /* no sm_100a device / feature not built */
    ALB_ERR_OOM = -6,
    ALB_ERR_NO_SLOT = -7,     /* KV cache: too few free cells for the ubatch */
};

/* ---------------------------------------------------------------- runtime */
ALB_API int          alb_version(void);
ALB_API const char * alb_last_error(void);
/* 0 when device `dev` is an sm_100 part this library can run on. */
ALB_API int          alb_device_check(int dev);
/* Device-side error word of the current device: 0, or the code of a bounded
 * in-kernel wait that expired (1 = mbarrier, 2 = cross-CTA / cross-rank flag),
 * or 3 = a decode step produced no valid next token (token 0 was fed back), or
 * 4 = alb_set_rows_f16 / alb_get_rows_f16 / alb_qk_norm_rope_kv_cells met a row
 * index out of range.
 * Kernels never trap; they record the error and return.  clear != 0 resets it. */
ALB_API int          alb_device_error(int clear);

/* ---------------------------------------------------------------- formats */
/* Bytes of the alb Q4_0 GPU layout of an [N x K] weight (K % 32 == 0), and of
 * one of its rows (0 for an invalid K). */
ALB_API size_t alb_q4_0_gpu_bytes(int64_t N, int64_t K);
ALB_API size_t alb_q4_0_row_bytes(int64_t K);
/* format_repack / repack<block_q4_0,4,4> (types.cpp:199-240): block_q4_0 rows
 * [N][K/32] (device) -> alb GPU layout (device). */
ALB_API int alb_repack_q4_0(void * dst, const void * src_blocks, int64_t N, int64_t K, void * stream);
/* inverse of alb_repack_q4_0 (tests / export) */
ALB_API int alb_unpack_q4_0(void * dst_blocks, const void * src, int64_t N, int64_t K, void * stream);

/* ----------------------------------------------------------- quantization */
/* quantize_row_q8_0 (arm.cpp:1819-1853) / nnml_quantize_mat_q8_0_4x4
 * (gemm.cpp:1943-2009): fp32 [rows][K] -> block_q8_0 [rows][K/32], RNE. */
ALB_API int alb_quantize_q8_0(const float * x, void * xq, int64_t K, int64_t rows, void * stream);

/* ------------------------------------------------------------------- GEMV */
/* nnml_gemv_q4_0_4x4_q8_0 (gemm.cpp:127-190) driven by forward_mul_mat
 * (arm.cpp:1855-1925), ne11 = 1: per row, acc = fma(float(I(n,b)),
 * f32(dx_b) * f32(dw_b), acc) over the blocks b in order from 0 (the NEON
 * chain, gemm.cpp:179-181), then y[n] = acc (+ residual[n] when non-null: the
 * ADD of qwen3.cpp:239/270 fused).  Bit-identical to the reference's
 * arithmetic.  W in the alb GPU layout (16-byte aligned), xq block_q8_0 [K/32];
 * K <= 12288. */
ALB_API int alb_gemv_q4_0_q8_0(const void * W, const void * xq, float * y, int64_t N, int64_t K,
                       const float * residual, void * stream);
/* forward_mul_mat_generic (common.cpp:120-248) with nnml_vec_dot_q4_0_q8_0
 * (arm.cpp:633-692), the path of the un-repacked lm head / token table: per
 * row, four partial block dots accumulated in two fp32 fma chains per lane
 * (even and odd blocks), summed as ((l0+l1)+(l2+l3)) per chain, then even +
 * odd, then the scalar tail of an odd block count.  y [N]. */
ALB_API int alb_mul_mat_q4_0_q8_0(const void * W, const void * xq, float * y, int64_t N, int64_t K, void * stream);
/* ------------------------------------------------------------------- GEMM */
/* nnml_gemm_q4_0_4x4_q8_0 (gemm.cpp:495-974) driven by forward_mul_mat
 * (arm.cpp:1855-1925), ne11 = M > 1 (prefill): every output the same fp32 fma
 * chain over the blocks as alb_gemv_q4_0_q8_0 (the reference's gemm and gemv
 * share it), + residual[m][n] when non-null; block dots on tcgen05 int8
 * tensor cores.  W in the alb GPU layout [N][K], xq block_q8_0 [M][K/32],
 * y / residual [M][N].  workspace: alb_gemm_workspace_bytes(M, K). */
ALB_API size_t alb_gemm_workspace_bytes(int64_t M, int64_t K);
ALB_API int alb_gemm_q4_0_q8_0(const void * W, const void * xq, float * y, int64_t M, int64_t N, int64_t K,
                               const float * residual, void * workspace, void * stream);
/* Debug twin of alb_gemv_q4_0_q8_0 writing the int32 block dots I[N][K/32]. */
ALB_API int alb_gemv_q4_0_q8_0_block_dots(const void * W, const void * xq, int32_t * I, int64_t N, int64_t K,
                                  void * stream);

/* ----------------------------------------------------------- elementwise */
/* RMS_NORM (ops.cpp:680-724; double sum of squares) followed by the graph's
 * MUL by w (binary.cpp:15-23, cgraph.cpp:115-120); w may be NULL.  x, y [rows][n]. */
ALB_API int alb_rms_norm(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps, void * stream);
/* swiglu_split (ops.cpp:1038-1092, arm.cpp:1789-1809): y = silu(g) * u. */
ALB_API int alb_swiglu(const float * g, const float * u, float * y, int64_t n, void * stream);
/* rms_norm_f32 + MUL (as alb_rms_norm) fused with quantize_row_q8_0
 * (arm.cpp:1819-1853) of the result: yq [rows][n/32] block_q8_0, the input of
 * the next mat-vec / mat-mul; y (fp32 result) may be NULL; n % 32 == 0. */
ALB_API int alb_rms_norm_q8(const float * x, const float * w, float * y, void * yq, int64_t rows, int64_t n,
                            float eps, void * stream);
/* alb_swiglu fused with quantize_row_q8_0 of the product (the down
 * projection's input); y may be NULL; n % 32 == 0. */
ALB_API int alb_swiglu_q8(const float * g, const float * u, float * y, void * yq, int64_t n, void * stream);
/* GET_ROWS of a Q4_0 table in the alb GPU layout (ops.cpp:12-52): out [n_ids][K]. */
ALB_API int alb_get_rows_q4_0(const void * W, int64_t n_rows, int64_t K, const int32_t * ids, int64_t n_ids,
                              float * out, void * stream);
/* SET_ROWS into fp16 (ops.cpp:135-181; cpy_k / cpy_v, cgraph.cpp:1114-1180):
 * dst[idx[r]][:] = fp16(src[r][:]) (round to nearest even) for r < n_rows; idx
 * (device, int64) are row indices of dst [dst_rows][row_len], e.g. the cell
 * indices of alb_kv_prepare.  row_len % 8 == 0, src and dst 16-byte aligned.  A
 * row whose index is outside [0, dst_rows) is skipped and alb_device_error()
 * reports 4. */
ALB_API int alb_set_rows_f16(const float * src, int64_t n_rows, int64_t row_len, const int64_t * idx, uint16_t * dst,
                             int64_t dst_rows, void * stream);
/* GET_ROWS of fp16 rows (ops.cpp:12-131 for an F16 source): dst[r][:] =
 * src[idx[r]][:] for r < n_rows, idx (device, int64) row indices of src
 * [src_rows][row_len].  With alb_kv_visible_cells it gathers the K/V cells one
 * sequence sees, in cell order, for alb_flash_attn (several sequences in one
 * cache).  row_len % 8 == 0, src and dst 16-byte aligned; an index outside
 * [0, src_rows) gives a zero row and alb_device_error() reports 4. */
ALB_API int alb_get_rows_f16(const uint16_t * src, int64_t src_rows, int64_t row_len, const int64_t * idx,
                             int64_t n_rows, uint16_t * dst, void * stream);
/* RoPE cos/sin table of nnml_rope_cache_init (ops.cpp:759-771; NEOX, ext_factor 0,
 * freq_scale 1): host-computed, copied to table_dev [max_pos][head_dim/2] (cos, sin). */
ALB_API int alb_rope_table(float * table_dev, int32_t max_pos, int32_t head_dim, float freq_base);
/* Per-head QK-RMSNorm * w + NEOX RoPE of Q and K and the fp16 KV store of K and V
 * (qwen3.cpp:215-224, ops.cpp:830-938, set_rows ops.cpp:135-181).  qkv [T][(Hq+2Hkv)*128]
 * fp32 (the fused QKV projection), q_out [T][Hq][128], caches [cells][Hkv][128] fp16;
 * token t is at position pos0+t.  head_dim is 128. */
ALB_API int alb_qk_norm_rope_kv(const float * qkv, int64_t T, int32_t n_head, int32_t n_head_kv,
                                const float * q_norm, const float * k_norm, float eps, const float * rope_table,
                                int32_t pos0, float * q_out, uint16_t * k_cache, uint16_t * v_cache, void * stream);

/* alb_qk_norm_rope_kv for a ubatch placed by the KV-cache manager: token t takes
 * position positions[t] (device int32; < max_pos, the RoPE table's rows) and
 * stores its K/V rows into cell cells[t] (device int64, e.g. alb_kv_prepare's
 * flat indices; < n_cells, the cache's rows).  A token outside those bounds is
 * skipped and alb_device_error() reports 4. */
ALB_API int alb_qk_norm_rope_kv_cells(const float * qkv, int64_t T, int32_t n_head, int32_t n_head_kv,
                                      const float * q_norm, const float * k_norm, float eps, const float * rope_table,
                                      int32_t max_pos, const int32_t * positions, const int64_t * cells,
                                      int64_t n_cells, float * q_out, uint16_t * k_cache, uint16_t * v_cache,
                                      void * stream);

/* ------------------------------------------------------------- attention */
/* nnml_compute_forward_flash_attn_ext_f16 (arm.cpp:2196-2433), one sequence,
 * causal: token t (position pos0+t) attends cells [0, pos0+t] of the fp16
 * caches [cells][Hkv][128]; GQA ratio n_head/n_head_kv in {1,2,4,8}.  Scores
 * are fp32 (Q rounded to fp16 as the reference), the softmax uses the global
 * max and the reference's NEON exp, and the sums of p and p*v are double in a
 * canonical order (cells in order within 128-cell chunks, chunk sums in chunk
 * order): the result does not depend on `splits` (the cells are split over that
 * many CTAs per KV head and token, whole chunks each, and merged in-kernel).
 * Workspace: alb_flash_attn_workspace_bytes(.., n_cells = pos0 + T) (no
 * state kept between calls); may be NULL when T > 1 and splits == 1 (the
 * token-tiled prefill kernel).  q/out [T][Hq][128]. */
ALB_API size_t alb_flash_attn_workspace_bytes(int32_t n_head, int32_t n_head_kv, int64_t T, int32_t splits,
                                             int32_t n_cells);
ALB_API int alb_flash_attn(const float * q, const uint16_t * k_cache, const uint16_t * v_cache, int64_t T,
                           int32_t n_head, int32_t n_head_kv, int32_t pos0, float scale, int32_t splits,
                           void * workspace, float * out, void * stream);

/* Size of the fixed device workspace of alb_flash_attn_static (one per device). */
#define ALB_FLASH_ATTN_STATIC_BYTES (4u << 20)
/* alb_flash_attn without a caller workspace and without allocating, for
 * callers that cannot call cudaMalloc: an nnml operator shim runs inside the
 * reference's graph walk with only params->work_data (host scratch) in hand
 * and no device allocator of its own.  The
 * workspace is a file-scope device array of ALB_FLASH_ATTN_STATIC_BYTES per
 * device (calls whose alb_flash_attn_workspace_bytes exceeds it return
 * ALB_ERR_INVALID).  Calls on one device share that array and must not
 * overlap in time.  The first call on a device looks the array up and clears
 * it (cudaGetSymbolAddress, cudaMemsetAsync on `stream`); make it outside any
 * stream capture.  The looked-up address is kept for the life of the process:
 * a cudaDeviceReset of that device is not supported afterwards.  Calls whose
 * path needs no workspace (T > 1 with one split: the token-tiled kernel) are
 * never rejected for size.  Same results as alb_flash_attn.  No counterpart in the
 * reference (its ops take scratch from params->work_data, thread.h:166-167). */
ALB_API int alb_flash_attn_static(const float * q, const uint16_t * k_cache, const uint16_t * v_cache, int64_t T,
                                  int32_t n_head, int32_t n_head_kv, int32_t pos0, float scale, int32_t splits,
                                  float * out, void * stream);

/* -------------------------------------------------------------- sampling */
/* sample_none (sampler.cpp:34-36): first index of the maximum of x[0..n).
 * scratch >= 1024 bytes, zeroed once before first use. */
ALB_API int alb_argmax(const float * x, int64_t n, void * scratch, int32_t * idx_out, void * stream);

/* ------------------------------------------------------- Qwen3 engine
 * llm_model + nnml_cgraph (build_qwen3_forward_tp, qwen3.cpp:174-275) +
 * llm_kv_cache + decoding_context (context.cpp:21-205) for one sequence, on
 * one GPU or as one tensor-parallel rank (one process/thread per GPU).  The
 * model is the seeded synthetic Qwen3 of the benchmark configs (weights
 * generated on the device; the same stream as oracle/oracle.c).  KV cache fp16,
 * greedy sampling. */
typedef struct alb_engine alb_engine;
typedef struct {
    int32_t n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff, n_vocab, tied;
    float   eps, freq_base;
} alb_qwen3_config;   /* llm_hparams subset (model.h), head_dim = key_length */

/* ncclGetUniqueId for tensor-parallel engines (128 bytes). */
ALB_API int alb_nccl_unique_id(void * out128);
/* Tensor-parallel communicator for the op-level ABI (NCCL, one per rank and
 * device).  The reference's GATHER of node partials (ops.cpp:1465-1511):
 * alb_allreduce_sum_f32 (dst = sum over ranks, NCCL's order) or
 * alb_allgather_f32 (dst [size][n], rank r's src at dst + r*n, for an ordered
 * sum on the device).  Stream-ordered; every rank makes the same calls. */
typedef struct alb_comm alb_comm;
ALB_API int alb_comm_create(const void * nccl_id, int32_t rank, int32_t size, int32_t device, alb_comm ** out);
ALB_API int alb_comm_destroy(alb_comm * comm);
ALB_API int alb_allreduce_sum_f32(alb_comm * comm, const float * src, float * dst, int64_t n, void * stream);
ALB_API int alb_allgather_f32(alb_comm * comm, const float * src, float * dst, int64_t n, void * stream);
/* al-gen.cpp:60-141 setup: weights, KV cache [max_ctx] and buffers for ubatches
 * of up to max_ubatch tokens on CUDA device `device`; tp_size > 1 joins the
 * NCCL clique `nccl_id` as tp_rank (n_head, n_head_kv, n_vocab divisible by
 * tp_size; n_ff by 32*tp_size). */
ALB_API int alb_engine_create(const alb_qwen3_config * cfg, uint64_t seed, int32_t max_ctx, int32_t max_ubatch,
                              int32_t tp_rank, int32_t tp_size, const void * nccl_id, int32_t device,
                              alb_engine ** out);
ALB_API int alb_engine_destroy(alb_engine * e);
ALB_API size_t alb_engine_device_bytes(const alb_engine * e);
/* llm_kv_cache::clear (cgraph.cpp:988-993): zero the KV cache. */
ALB_API int alb_engine_reset(alb_engine * e);
/* decode() over a prompt chunk at positions [pos0, pos0+n) in ubatches of
 * max_ubatch; returns the greedy next token. */
ALB_API int alb_engine_prefill(alb_engine * e, const int32_t * tokens, int32_t n, int32_t pos0, int32_t * next_token);
/* One greedy decode step of `token` at position `pos` (one CUDA-graph replay). */
ALB_API int alb_engine_decode(alb_engine * e, int32_t token, int32_t pos, int32_t * next_token);
/* n_steps greedy steps without host round trips; tokens_out (nullable) gets the
 * generated tokens; sync != 0 waits for completion. */
ALB_API int alb_engine_decode_loop(alb_engine * e, int32_t token, int32_t pos, int32_t n_steps, int32_t * tokens_out,
                                   int32_t sync);
/* Last logits of this rank's vocabulary shard [n_vocab / tp_size]. */
ALB_API int alb_engine_logits(alb_engine * e, float * host, int64_t n);
/* The residual stream (the hidden state before the output norm) of the last
 * forward pass, rows [0, rows) of its ubatch, [rows][n_embd] (host). */
ALB_API int alb_engine_hidden(alb_engine * e, float * host, int64_t rows);
/* info[0..7] = local vocab, vocab offset, local q heads, local kv heads, local
 * ffn, kernel launches per decode step, device bytes, decode attention splits */
ALB_API int alb_engine_info(const alb_engine * e, int64_t * info, int32_t n);
ALB_API void * alb_engine_stream(alb_engine * e);
/* This rank's shard of weight (layer, kind) in block_q4_0 rows (host), kinds as
 * oracle.h (4 WQ, 5 WK, 6 WV, 7 WO, 11 GATE, 12 UP, 13 DOWN; layer -1 kind 0 =
 * token table, kind 1 = untied lm head).  host = NULL only reports the shard shape. */
ALB_API int alb_engine_weight_blocks(alb_engine * e, int32_t layer, int32_t kind, void * host, int64_t * rows,
                                     int64_t * cols);
ALB_API int alb_engine_norm_weights(alb_engine * e, int32_t layer, int32_t kind, float * host, int64_t n);
/* External weights (the reference's model load, model.cpp:355-474 with
 * slice_tensor, model.cpp:40-110): host = the FULL tensor of (layer, kind) in
 * block_q4_0 rows (all ranks' rows / columns: rows x cols values); the engine
 * keeps its tensor-parallel shard (Q, K, V, gate, up, untied lm head by rows;
 * O, down by columns; the token table whole) and repacks it on the device.
 * Kinds as alb_engine_weight_blocks, plus layer -1 kind 1 = untied lm head. */
ALB_API int alb_engine_set_weight_blocks(alb_engine * e, int32_t layer, int32_t kind, const void * host, int64_t rows,
                                         int64_t cols);
/* fp32 norm weights of (layer, kind): 3 attn, 10 ffn (n_embd), 8 q, 9 k (head_dim);
 * layer -1 kind 2 = output norm. */
ALB_API int alb_engine_set_norm_weights(alb_engine * e, int32_t layer, int32_t kind, const float * host, int64_t n);
/* Measurement hook: mean duration and algorithmic bytes per launch of the
 * decode step's Q4_0 mat-vecs replayed alone from a CUDA graph. */
ALB_API int alb_engine_time_gemv(alb_engine * e, int32_t reps, float * us_per_launch, double * bytes_per_launch);
/* Measurement hook: mean duration and int8 operations per launch of the prefill
 * mat-muls of one max_ubatch-token ubatch (all layers) replayed alone from a CUDA graph. */
ALB_API int alb_engine_time_prefill_gemm(alb_engine * e, int32_t reps, float * us_per_launch, double * ops_per_launch);
/* Fill every layer's KV cache for positions [0, n_pos) with seeded N(0,1) fp16. */
ALB_API int alb_engine_fill_kv(alb_engine * e, int32_t n_pos, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif /* ALB_CUDA_H */
