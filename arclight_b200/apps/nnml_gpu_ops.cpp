// nnml_gpu_ops: the reference's decode-path operators as GPU operators over
// libalb_cuda.so (see nnml_gpu_ops.h for the calling shape).
#include "nnml_gpu_ops.h"

#include <cstring>

namespace {

// Only thread 0 of the group launches (the whole operator is one launch).
inline bool not_mine(const nnml_gpu_state * p) { return p && p->ith != 0; }

inline float param_f32(const nnml_gpu_tensor * t, int i) {
    float v;
    std::memcpy(&v, &t->op_params[i], sizeof v);
    return v;
}

// Contiguous fp32 rows of n elements: the kernels take dense [rows][n].
inline bool dense_f32(const nnml_gpu_tensor * t) {
    return t && t->data && t->nb[0] == 4 && t->nb[1] == (size_t)t->ne[0] * 4;
}

}  // namespace

extern "C" int nnml_gpu_forward_mul_mat(const nnml_gpu_state * params, nnml_gpu_tensor * dst) {
    if (!params || !dst) return ALB_ERR_INVALID;
    if (not_mine(params)) return ALB_OK;
    const nnml_gpu_tensor * w = dst->src[0], * x = dst->src[1];
    if (!w || !x || !w->data || !x->data || !dst->data) return ALB_ERR_INVALID;
    const int64_t K = w->ne[0], N = w->ne[1];
    if (x->ne[0] != K || x->ne[1] != 1 || dst->ne[0] != N) return ALB_ERR_INVALID;   // one activation row
    if (!params->xq || params->xq_bytes < (size_t)(K / 32) * 34) return ALB_ERR_INVALID;
    int rc = alb_quantize_q8_0(static_cast<const float *>(x->data), params->xq, K, 1, params->stream);
    if (rc != ALB_OK) return rc;
    if (dst->op_params[0] == 1)   // repacked weight: the 4x4 gemv chain
        return alb_gemv_q4_0_q8_0(w->data, params->xq, static_cast<float *>(dst->data), N, K, nullptr, params->stream);
    return alb_mul_mat_q4_0_q8_0(w->data, params->xq, static_cast<float *>(dst->data), N, K, params->stream);
}

extern "C" int nnml_gpu_forward_rms_norm_mul(const nnml_gpu_state * params, nnml_gpu_tensor * dst) {
    if (!params || !dst) return ALB_ERR_INVALID;
    if (not_mine(params)) return ALB_OK;
    const nnml_gpu_tensor * x = dst->src[0], * w = dst->src[1];
    if (!dense_f32(x) || !dense_f32(dst) || (w && !w->data)) return ALB_ERR_INVALID;
    if (dst->ne[0] != x->ne[0] || dst->ne[1] != x->ne[1] || (w && w->ne[0] != x->ne[0])) return ALB_ERR_INVALID;
    return alb_rms_norm(static_cast<const float *>(x->data), w ? static_cast<const float *>(w->data) : nullptr,
                        static_cast<float *>(dst->data), x->ne[1], x->ne[0], param_f32(dst, 0), params->stream);
}

extern "C" int nnml_gpu_forward_get_rows(const nnml_gpu_state * params, nnml_gpu_tensor * dst) {
    if (!params || !dst) return ALB_ERR_INVALID;
    if (not_mine(params)) return ALB_OK;
    const nnml_gpu_tensor * table = dst->src[0], * ids = dst->src[1];
    if (!table || !ids || !table->data || !ids->data || !dense_f32(dst)) return ALB_ERR_INVALID;
    if (dst->ne[0] != table->ne[0] || dst->ne[1] != ids->ne[0]) return ALB_ERR_INVALID;
    return alb_get_rows_q4_0(table->data, table->ne[1], table->ne[0], static_cast<const int32_t *>(ids->data),
                             ids->ne[0], static_cast<float *>(dst->data), params->stream);
}

extern "C" int nnml_gpu_forward_set_rows(const nnml_gpu_state * params, nnml_gpu_tensor * dst) {
    if (!params || !dst) return ALB_ERR_INVALID;
    if (not_mine(params)) return ALB_OK;
    const nnml_gpu_tensor * rows = dst->src[0], * idx = dst->src[1];
    if (!rows || !idx || !idx->data || !dense_f32(rows) || !dst->data) return ALB_ERR_INVALID;
    // dst: dense fp16 rows of the same length as src0's
    if (dst->ne[0] != rows->ne[0] || dst->nb[0] != 2 || dst->nb[1] != (size_t)dst->ne[0] * 2) return ALB_ERR_INVALID;
    if (idx->ne[0] != rows->ne[1] || idx->nb[0] != 8) return ALB_ERR_INVALID;
    return alb_set_rows_f16(static_cast<const float *>(rows->data), rows->ne[1], rows->ne[0],
                            static_cast<const int64_t *>(idx->data), static_cast<uint16_t *>(dst->data), dst->ne[1],
                            params->stream);
}

extern "C" int nnml_gpu_forward_swiglu(const nnml_gpu_state * params, nnml_gpu_tensor * dst) {
    if (!params || !dst) return ALB_ERR_INVALID;
    if (not_mine(params)) return ALB_OK;
    const nnml_gpu_tensor * g = dst->src[0], * u = dst->src[1];
    if (!dense_f32(g) || !dense_f32(u) || !dense_f32(dst)) return ALB_ERR_INVALID;
    const int64_t n = dst->ne[0] * dst->ne[1];
    if (g->ne[0] * g->ne[1] != n || u->ne[0] * u->ne[1] != n) return ALB_ERR_INVALID;
    return alb_swiglu(static_cast<const float *>(g->data), static_cast<const float *>(u->data),
                      static_cast<float *>(dst->data), n, params->stream);
}

extern "C" int nnml_gpu_forward_flash_attn_ext(const nnml_gpu_state * params, nnml_gpu_tensor * dst) {
    if (!params || !dst) return ALB_ERR_INVALID;
    if (not_mine(params)) return ALB_OK;
    const nnml_gpu_tensor * q = dst->src[0], * k = dst->src[1], * v = dst->src[2];
    if (!q || !k || !v || !q->data || !k->data || !v->data || !dst->data) return ALB_ERR_INVALID;
    if (q->ne[0] != 128 || k->ne[0] != 128 || v->ne[0] != 128) return ALB_ERR_INVALID;   // head_dim 128
    const int64_t T = q->ne[2];
    const int32_t n_head = (int32_t)q->ne[1], n_head_kv = (int32_t)k->ne[1];
    const int32_t pos0 = dst->op_params[0], splits = dst->op_params[2] > 0 ? dst->op_params[2] : 1;
    const size_t need = alb_flash_attn_workspace_bytes(n_head, n_head_kv, T, splits, pos0 + (int32_t)T);
    void * ws = params->attn_ws;
    if (need > params->attn_ws_bytes) {
        if (!(T > 1 && splits == 1)) return ALB_ERR_INVALID;   // only the token-tiled prefill path needs none
        ws = nullptr;
    }
    return alb_flash_attn(static_cast<const float *>(q->data), static_cast<const uint16_t *>(k->data),
                          static_cast<const uint16_t *>(v->data), T, n_head, n_head_kv, pos0, param_f32(dst, 1),
                          splits, ws, static_cast<float *>(dst->data), params->stream);
}

extern "C" int nnml_gpu_sample_greedy(const nnml_gpu_state * params, nnml_gpu_tensor * dst) {
    if (!params || !dst) return ALB_ERR_INVALID;
    if (not_mine(params)) return ALB_OK;
    const nnml_gpu_tensor * logits = dst->src[0];
    if (!logits || !logits->data || !dst->data || !params->attn_ws || params->attn_ws_bytes < 1024)
        return ALB_ERR_INVALID;
    return alb_argmax(static_cast<const float *>(logits->data), logits->ne[0], params->attn_ws,
                      static_cast<int32_t *>(dst->data), params->stream);
}
