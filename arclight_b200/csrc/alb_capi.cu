// C ABI wrappers of the elementwise / attention / sampling kernels.
#include <cmath>
#include <vector>

#include "alb_common.cuh"
#include "alb_internal.h"

using namespace alb;

extern "C" int alb_rms_norm(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps,
                            void * stream) {
    ALB_CHECK_ARG(x && y && rows > 0 && n > 0 && eps >= 0.0f);
    ALB_CUDA_TRY(launch_rms_norm(x, w, y, rows, n, eps, true, (cudaStream_t)stream));
    return ALB_OK;
}

extern "C" int alb_swiglu(const float * g, const float * u, float * y, int64_t n, void * stream) {
    ALB_CHECK_ARG(g && u && y && n > 0);
    ALB_CUDA_TRY(launch_swiglu(g, u, y, n, true, (cudaStream_t)stream));
    return ALB_OK;
}

extern "C" int alb_rms_norm_q8(const float * x, const float * w, float * y, void * yq, int64_t rows, int64_t n,
                               float eps, void * stream) {
    ALB_CHECK_ARG(x && yq && rows > 0 && rows < (1LL << 31) && n > 0 && n % 32 == 0 && n / 256 < 65535 && eps >= 0.0f);
    ALB_CUDA_TRY(launch_rms_norm_q8(x, w, y, yq, rows, n, eps, true, (cudaStream_t)stream));
    return ALB_OK;
}

extern "C" int alb_swiglu_q8(const float * g, const float * u, float * y, void * yq, int64_t n, void * stream) {
    ALB_CHECK_ARG(g && u && yq && n > 0 && n % 32 == 0 && n / 32 < (1LL << 34));
    ALB_CUDA_TRY(launch_swiglu_q8(g, u, y, yq, n, true, (cudaStream_t)stream));
    return ALB_OK;
}

extern "C" int alb_get_rows_q4_0(const void * W, int64_t n_rows, int64_t K, const int32_t * ids, int64_t n_ids,
                                 float * out, void * stream) {
    ALB_CHECK_ARG(W && ids && out && n_rows > 0 && K > 0 && K % 32 == 0 && n_ids > 0 && n_ids < (1 << 30));
    ALB_CUDA_TRY(launch_embed((const uint8_t *)W, n_rows, K, ids, (int)n_ids, out, nullptr, true, (cudaStream_t)stream));
    return ALB_OK;
}

// SET_ROWS of fp32 rows into an fp16 row array at device indices (the KV store
// of cpy_k / cpy_v with the KV-cache manager's cell indices).
extern "C" int alb_set_rows_f16(const float * src, int64_t n_rows, int64_t row_len, const int64_t * idx, uint16_t * dst,
                                int64_t dst_rows, void * stream) {
    ALB_CHECK_ARG(src && idx && dst && n_rows > 0 && row_len > 0 && row_len % 8 == 0 && dst_rows > 0);
    ALB_CHECK_ARG(n_rows <= ((int64_t)1 << 40) / row_len && dst_rows <= ((int64_t)1 << 40) / row_len);
    ALB_CHECK_ARG(((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 15) == 0);
    ALB_CUDA_TRY(alb::launch_set_rows_f16(src, n_rows, row_len, idx, dst, dst_rows, (cudaStream_t)stream));
    return ALB_OK;
}

// GET_ROWS of fp16 rows at device indices (e.g. the KV cells one sequence sees,
// gathered for attention).
extern "C" int alb_get_rows_f16(const uint16_t * src, int64_t src_rows, int64_t row_len, const int64_t * idx,
                                int64_t n_rows, uint16_t * dst, void * stream) {
    ALB_CHECK_ARG(src && idx && dst && n_rows > 0 && src_rows > 0 && row_len > 0 && row_len % 8 == 0);
    ALB_CHECK_ARG(n_rows <= ((int64_t)1 << 40) / row_len && src_rows <= ((int64_t)1 << 40) / row_len);
    ALB_CHECK_ARG(((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 15) == 0);
    ALB_CUDA_TRY(alb::launch_get_rows_f16(src, src_rows, row_len, idx, n_rows, dst, (cudaStream_t)stream));
    return ALB_OK;
}

namespace alb {
// nnml_rope_cache_init (ops.cpp:759-771) with ext_factor 0, freq_scale 1,
// mscale 1: theta_0 = p, theta_{i+1} = theta_i * theta_scale (fp32 products),
// theta_scale = powf(freq_base, -2/n_dims) (ops.cpp:886).
void rope_table_host(std::vector<float> & t, int32_t max_pos, int32_t head_dim, float freq_base) {
    const int half = head_dim / 2;
    t.assign((size_t)max_pos * half * 2, 0.0f);
    const float theta_scale = powf(freq_base, -2.0f / (float)head_dim);
    for (int32_t p = 0; p < max_pos; ++p) {
        float theta = (float)p;
        for (int i = 0; i < half; ++i) {
            t[((size_t)p * half + i) * 2 + 0] = cosf(theta);
            t[((size_t)p * half + i) * 2 + 1] = sinf(theta);
            theta *= theta_scale;
        }
    }
}
}  // namespace alb

extern "C" int alb_rope_table(float * table_dev, int32_t max_pos, int32_t head_dim, float freq_base) {
    ALB_CHECK_ARG(table_dev && max_pos > 0 && head_dim == 128 && freq_base > 0.0f);
    std::vector<float> t;
    rope_table_host(t, max_pos, head_dim, freq_base);
    ALB_CUDA_TRY(cudaMemcpy(table_dev, t.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice));
    return ALB_OK;
}

extern "C" int alb_qk_norm_rope_kv(const float * qkv, int64_t T, int32_t n_head, int32_t n_head_kv,
                                   const float * q_norm, const float * k_norm, float eps, const float * rope_table,
                                   int32_t pos0, float * q_out, uint16_t * k_cache, uint16_t * v_cache,
                                   void * stream) {
    ALB_CHECK_ARG(qkv && q_norm && k_norm && rope_table && q_out && k_cache && v_cache);
    ALB_CHECK_ARG(T > 0 && T < 65536 && n_head > 0 && n_head_kv > 0 && pos0 >= 0);
    QkvArgs a;
    a.qkv = qkv; a.qkv_stride = (int64_t)(n_head + 2 * n_head_kv) * 128;
    a.Hq = n_head; a.Hkv = n_head_kv; a.T = (int)T;
    a.q_norm = q_norm; a.k_norm = k_norm; a.eps = eps;
    a.rope = reinterpret_cast<const float2 *>(rope_table);
    a.pos0 = pos0; a.q_out = q_out; a.kc = k_cache; a.vc = v_cache; a.pdl = true;
    ALB_CUDA_TRY(launch_qk_norm_rope_kv(a, (cudaStream_t)stream));
    return ALB_OK;
}

// The same with per-token positions and cells (device arrays), for a ubatch
// placed by the KV-cache manager (several sequences, cells != positions).
extern "C" int alb_qk_norm_rope_kv_cells(const float * qkv, int64_t T, int32_t n_head, int32_t n_head_kv,
                                         const float * q_norm, const float * k_norm, float eps,
                                         const float * rope_table, int32_t max_pos, const int32_t * positions,
                                         const int64_t * cells, int64_t n_cells, float * q_out, uint16_t * k_cache,
                                         uint16_t * v_cache, void * stream) {
    ALB_CHECK_ARG(qkv && q_norm && k_norm && rope_table && q_out && k_cache && v_cache && positions && cells);
    ALB_CHECK_ARG(T > 0 && T < 65536 && n_head > 0 && n_head_kv > 0 && max_pos > 0 && n_cells > 0);
    QkvArgs a;
    a.qkv = qkv; a.qkv_stride = (int64_t)(n_head + 2 * n_head_kv) * 128;
    a.Hq = n_head; a.Hkv = n_head_kv; a.T = (int)T;
    a.q_norm = q_norm; a.k_norm = k_norm; a.eps = eps;
    a.rope = reinterpret_cast<const float2 *>(rope_table);
    a.q_out = q_out; a.kc = k_cache; a.vc = v_cache; a.pdl = true;
    a.pos_tok = positions; a.cell_tok = cells; a.n_cells = n_cells; a.max_pos = max_pos;
    ALB_CUDA_TRY(launch_qk_norm_rope_kv(a, (cudaStream_t)stream));
    return ALB_OK;
}

extern "C" size_t alb_flash_attn_workspace_bytes(int32_t n_head, int32_t n_head_kv, int64_t T, int32_t splits,
                                                 int32_t n_cells) {
    if (n_head <= 0 || n_head_kv <= 0 || T <= 0 || splits <= 0 || n_cells <= 0) return 0;
    return flash_attn_ws_bytes(n_head, n_head_kv, (int)T, splits, n_cells);
}

extern "C" int alb_flash_attn(const float * q, const uint16_t * k_cache, const uint16_t * v_cache, int64_t T,
                              int32_t n_head, int32_t n_head_kv, int32_t pos0, float scale, int32_t splits,
                              void * workspace, float * out, void * stream) {
    ALB_CHECK_ARG(q && k_cache && v_cache && out && T > 0 && T < 65536 && pos0 >= 0);
    ALB_CHECK_ARG(n_head > 0 && n_head_kv > 0 && n_head % n_head_kv == 0);
    const int G = n_head / n_head_kv;
    ALB_CHECK_ARG(G == 1 || G == 2 || G == 4 || G == 8);
    ALB_CHECK_ARG(splits >= 1 && splits <= 65535 && (int64_t)pos0 + T < (int64_t)1 << 30);
    FlashArgs f;
    f.ncap = (int)(pos0 + T);
    f.q = q; f.kc = k_cache; f.vc = v_cache; f.Hq = n_head; f.Hkv = n_head_kv; f.T = (int)T;
    f.pos0 = pos0; f.scale = scale; f.S = splits; f.ws = (float *)workspace; f.out = out; f.pdl = true;
    ALB_CHECK_ARG(workspace || !flash_attn_uses_ws(n_head, n_head_kv, (int)T, splits, f.ncap));
    ALB_CUDA_TRY(launch_flash_attn(f, (cudaStream_t)stream));
    return ALB_OK;
}

extern "C" int alb_argmax(const float * x, int64_t n, void * scratch, int32_t * idx_out, void * stream) {
    ALB_CHECK_ARG(x && scratch && idx_out && n > 0 && n < (int64_t)0x7FFFFFFF);
    ALB_CUDA_TRY(launch_argmax(x, n, 0, scratch, nullptr, idx_out, true, (cudaStream_t)stream));
    return ALB_OK;
}
