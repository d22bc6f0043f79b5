/*
 * KV-cache cell manager (host side) of the ArcLight B200 path.
 *
 * Replaces the slot and cell bookkeeping of the reference's llm_kv_cache /
 * llm_kv_cells (nnml/include/cgraph.h:249-374, 612-1046; nnml/src/cgraph.cpp:
 * 915-1600): which cache cell every token of a ubatch writes its K/V row to,
 * which cells each query row may attend to, and the per-sequence position
 * bookkeeping (removal, shifts, min/max).  The K/V rows themselves live on the
 * device (alb_engine's cache, or any [n_stream * kv_size] row array); this
 * object only computes indices and masks, identical to the reference's for the
 * same sequence of calls.
 *
 * Ubatches are given as flat arrays: n_tokens positions and one sequence id per
 * token.  Their distinct sequence ids, ascending, are the ubatch's sequence set
 * (llm_ubatch::seq_id_unq).  With one stream per sequence (unified = 0) the
 * tokens must come as equal runs, one run per sequence in that order (the
 * reference's split_equal ubatches).
 *
 * Cell indices handed out and taken back are flat: stream * kv_size + cell, the
 * reference's K/V row indices (set_inputs_attn_kidx, cgraph.cpp:1182-1194).
 *
 * Host memory only, no CUDA call.  A cache object has one owner: calls on one
 * object must not overlap; calls on distinct objects are independent.  Errors
 * leave the cells unchanged and return ALB_ERR_INVALID (message in
 * alb_last_error()), where the reference asserts.
 */
#ifndef ALB_KVCACHE_H
#define ALB_KVCACHE_H

#include <stdint.h>

#include "alb_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* LLM_MAX_SEQ (cgraph.h:26): sequence ids are 0..63 */
#define ALB_KV_MAX_SEQ 64
/* NNML_KQ_MASK_PAD (cgraph.h:28): mask rows per stream are padded to 64 */
#define ALB_KV_MASK_PAD 64

typedef struct alb_kv_cache alb_kv_cache;

/* llm_kv_cache::llm_kv_cache (cgraph.cpp:915-986), cells only: kv_size cells
 * per stream, n_stream = unified ? 1 : n_seq_max; kv_size % n_pad == 0. */
ALB_API int alb_kv_create(uint32_t kv_size, uint32_t n_seq_max, int32_t unified, uint32_t n_pad,
                          alb_kv_cache ** out);
ALB_API int alb_kv_destroy(alb_kv_cache * kv);
/* llm_kv_cache::clear (cgraph.cpp:988-993): every cell empty, heads at 0. */
ALB_API int alb_kv_clear(alb_kv_cache * kv);

/* llm_kv_cache::find_slot (cgraph.cpp:1317-1418) without changing any cell:
 * idxs_out[n_tokens] gets the cell of every token.  ALB_ERR_NO_SLOT when the
 * stream has too few free cells (cont != 0: too few contiguous ones). */
ALB_API int alb_kv_find_slot(const alb_kv_cache * kv, const int32_t * pos, const int32_t * seq_id, int32_t n_tokens,
                             int32_t cont, int64_t * idxs_out);
/* llm_kv_cache::prepare (cgraph.cpp:1263-1315): slots for n_ubatches ubatches
 * placed one after another (ubatch u has sizes[u] tokens; pos / seq_id hold
 * them back to back), then every cell restored.  All or nothing: on
 * ALB_ERR_NO_SLOT idxs_out is untouched and the cells are as before. */
ALB_API int alb_kv_prepare(alb_kv_cache * kv, const int32_t * sizes, int32_t n_ubatches, const int32_t * pos,
                           const int32_t * seq_id, int64_t * idxs_out);
/* llm_kv_cache::apply / apply_ubatch / get_n_kv (cgraph.cpp:1420-1492): place
 * the ubatch in the cells idxs (from prepare or find_slot); n_kv_out (nullable)
 * gets the cells the attention must cover: max(n_pad, used cells rounded up to
 * n_pad), at most kv_size. */
ALB_API int alb_kv_apply(alb_kv_cache * kv, const int32_t * pos, const int32_t * seq_id, int32_t n_tokens,
                         const int64_t * idxs, uint32_t * n_kv_out);
/* llm_kv_cache::seq_rm (cgraph.cpp:1535-1592): drop seq_id (-1: every
 * sequence) from the cells at positions [p0, p1) (p0 < 0: 0; p1 < 0: no end). */
ALB_API int alb_kv_seq_rm(alb_kv_cache * kv, int32_t seq_id, int32_t p0, int32_t p1);
/* llm_kv_cache::seq_add (cgraph.cpp:1501-1533): positions [p0, p1) of seq_id
 * move by shift; cells whose position turns negative are freed. */
ALB_API int alb_kv_seq_add(alb_kv_cache * kv, int32_t seq_id, int32_t p0, int32_t p1, int32_t shift);
/* llm_kv_cache::seq_pos_min / seq_pos_max (cgraph.cpp:1008-1018): -1 when the
 * sequence holds no cell. */
ALB_API int alb_kv_seq_pos_range(const alb_kv_cache * kv, int32_t seq_id, int32_t * pos_min, int32_t * pos_max);
/* llm_kv_cache::set_inputs_attn_mask (cgraph.cpp:1224-1261): the fp32 mask
 * [n_stream_ub][pad(n_tokens / n_stream_ub, 64)][n_kv] of one ubatch: 0 where
 * query token i may see cell j (same sequence, position <= its own), -INFINITY
 * elsewhere and on the padding rows. */
ALB_API int alb_kv_mask(const alb_kv_cache * kv, const int32_t * pos, const int32_t * seq_id, int32_t n_tokens,
                        int32_t n_stream_ub, uint32_t n_kv, float * mask);
/* One row of that mask as a list: the flat indices (stream * kv_size + cell,
 * ascending) of the cells j < n_kv that query (seq_id, pos) may see, into
 * cells_out (room for n_kv); *n_out = their count.  Gathering those K/V rows
 * (alb_get_rows_f16) gives the contiguous cache alb_flash_attn takes. */
ALB_API int alb_kv_visible_cells(const alb_kv_cache * kv, int32_t seq_id, int32_t pos, uint32_t n_kv,
                                 int64_t * cells_out, int32_t * n_out);
/* Inspection: cell `cell` of stream `stream`: its position (-1 empty), the
 * bit set of its sequences and its accumulated shift. */
ALB_API int alb_kv_cell(const alb_kv_cache * kv, uint32_t stream, uint32_t cell, int32_t * pos, uint64_t * seqs,
                        int32_t * shift);
/* info[0..5] = kv_size, n_stream, n_pad, used cells of `stream`, its head,
 * its last used cell + 1 */
ALB_API int alb_kv_info(const alb_kv_cache * kv, uint32_t stream, int64_t * info, int32_t n);

#ifdef __cplusplus
}
#endif
#endif /* ALB_KVCACHE_H */
