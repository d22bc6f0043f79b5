// Driver for the reference's own portable nnml code (oracle/_ref build only).
// Each ref_* entry builds nnml tensors with the reference's constructors and
// runs the reference's own nnml_compute_forward_* / quantizer on them, single
// threaded.  tests/golden/make_golden.py calls these through ctypes to write
// the golden fixtures that pin oracle/oracle.c.  Test infrastructure only.
#include <cstdint>
#include <cstring>
#include <vector>

#include "memory.h"
#include "ops.h"
#include "tensor.h"
#include "thread.h"

namespace {
nnml_memory_t make_mem(size_t bytes) {
    nnml_memory::cparams p;
    p.strategy = NNML_ALLOC_STRATEGY_UMA;
    p.n_nodes_manual = 1;
    p.total_wsize_bytes = bytes;
    p.total_csize_bytes = bytes;
    p.total_kvsize_bytes = 1 << 20;
    p.tmp_work_size_bytes = 1 << 20;
    p.zero_init = true;
    return nnml_memory::create(p);
}
struct state {
    std::vector<uint8_t> work;
    nnml_compute_state st;
    state() : work(4 << 20) { st.ith = 0; st.nth = 1; st.ith_global = 0; st.nth_global = 1; st.work_size = work.size(); st.work_data = work.data(); }
};
}  // namespace

extern "C" {

void ref_quantize_row_q4_0(const float * x, void * y, int64_t k) { quantize_row_q4_0_ref(x, (block_q4_0 *)y, k); }
void ref_dequantize_row_q4_0(const void * x, float * y, int64_t k) { dequantize_row_q4_0((const block_q4_0 *)x, y, k); }
void ref_quantize_row_q8_0_ref(const float * x, void * y, int64_t k) { quantize_row_q8_0_ref(x, (block_q8_0 *)y, k); }
void ref_dequantize_row_q8_0(const void * x, float * y, int64_t k) { dequantize_row_q8_0((const block_q8_0 *)x, y, k); }
uint16_t ref_fp32_to_fp16(float f) { return nnml_compute_fp32_to_fp16(f); }
float ref_fp16_to_fp32(uint16_t h) { return nnml_compute_fp16_to_fp32(h); }

// repack<block_q4_0, 4, 4> (types.cpp:199-201) on a [k x nrow] Q4_0 weight tensor
int ref_repack_q4_0_4x4(const void * src, void * dst, int64_t nrow, int64_t k) {
    const size_t bytes = (size_t)nrow * (k / 32) * sizeof(block_q4_0);
    auto mem = make_mem(bytes * 2 + (1 << 20));
    nnml_tensor * t = nnml_tensor::new_2d(mem, NNML_TENSOR_TYPE_WEIGHT, 0, 0, NNML_TYPE_Q4_0, k, nrow);
    const int rc = repack<block_q4_0, 4, 4>(t, src, bytes);
    memcpy(dst, t->tensor_data(), bytes);
    return rc;
}

// RMS_NORM (ops.cpp:680-724) followed by MUL with the [n] weight (binary.cpp)
void ref_rms_norm_mul(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps) {
    auto mem = make_mem((size_t)rows * n * 4 * 4 + (1 << 20));
    state s;
    nnml_tensor * a = nnml_tensor::new_2d(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, NNML_TYPE_F32, n, rows);
    memcpy(a->tensor_data(), x, (size_t)rows * n * 4);
    nnml_tensor * node = nnml_rms_norm(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, a, eps);
    nnml_compute_forward_rms_norm(node, &s.st);
    nnml_tensor * out = node;
    if (w) {
        nnml_tensor * wt = nnml_tensor::new_1d(mem, NNML_TENSOR_TYPE_WEIGHT, 0, 0, NNML_TYPE_F32, n);
        memcpy(wt->tensor_data(), w, (size_t)n * 4);
        out = nnml_mul(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, node, wt);
        nnml_compute_forward_mul(out, &s.st);
    }
    memcpy(y, out->tensor_data(), (size_t)rows * n * 4);
}

// ROPE NEOX (ops.cpp:830-961) on x [T][n_heads][head_dim], positions pos[T]
void ref_rope_neox(const float * x, float * y, int64_t n_heads, int64_t head_dim, int64_t T,
                   const int32_t * pos, float freq_base) {
    auto mem = make_mem((size_t)T * n_heads * head_dim * 4 * 3 + (1 << 20));
    state s;
    nnml_tensor * a = nnml_tensor::new_3d(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, NNML_TYPE_F32, head_dim, n_heads, T);
    memcpy(a->tensor_data(), x, (size_t)T * n_heads * head_dim * 4);
    nnml_tensor * p = nnml_tensor::new_1d(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, NNML_TYPE_I32, T);
    memcpy(p->tensor_data(), pos, (size_t)T * 4);
    nnml_tensor * node = nnml_rope_ext(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, a, p, nullptr, (int)head_dim,
                                       NNML_ROPE_TYPE_NEOX, 40960, freq_base, 1.0f, 0.0f, 1.0f, 32.0f, 1.0f);
    nnml_compute_forward_rope(node, &s.st);
    memcpy(y, node->tensor_data(), (size_t)T * n_heads * head_dim * 4);
}

// GET_ROWS on a Q4_0 [cols x rows] table (ops.cpp:12-52)
void ref_get_rows_q4_0(const void * table, int64_t rows, int64_t cols, const int32_t * ids, int64_t n_ids, float * out) {
    const size_t bytes = (size_t)rows * (cols / 32) * sizeof(block_q4_0);
    auto mem = make_mem(bytes + (size_t)n_ids * cols * 4 + (1 << 20));
    state s;
    nnml_tensor * t = nnml_tensor::new_2d(mem, NNML_TENSOR_TYPE_WEIGHT, 0, 0, NNML_TYPE_Q4_0, cols, rows);
    memcpy(t->tensor_data(), table, bytes);
    nnml_tensor * i = nnml_tensor::new_1d(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, NNML_TYPE_I32, n_ids);
    memcpy(i->tensor_data(), ids, (size_t)n_ids * 4);
    nnml_tensor * node = nnml_get_rows(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, t, i);
    nnml_compute_forward_get_rows(node, &s.st);
    memcpy(out, node->tensor_data(), (size_t)n_ids * cols * 4);
}

// SET_ROWS fp32 -> fp16 cache rows (ops.cpp:135-181, cgraph.cpp:1114-1180)
void ref_set_rows_f16(uint16_t * cache, int64_t n_cells, int64_t n, const float * src, const int64_t * idx, int64_t n_rows) {
    auto mem = make_mem((size_t)n_cells * n * 2 + (size_t)n_rows * n * 4 + (1 << 20));
    state s;
    nnml_tensor * c = nnml_tensor::new_2d(mem, NNML_TENSOR_TYPE_KVCACHE, 0, 0, NNML_TYPE_F16, n, n_cells);
    memcpy(c->tensor_data(), cache, (size_t)n_cells * n * 2);
    nnml_tensor * a = nnml_tensor::new_2d(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, NNML_TYPE_F32, n, n_rows);
    memcpy(a->tensor_data(), src, (size_t)n_rows * n * 4);
    nnml_tensor * i = nnml_tensor::new_1d(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, NNML_TYPE_I64, n_rows);
    memcpy(i->tensor_data(), idx, (size_t)n_rows * 8);
    nnml_tensor * node = nnml_set_rows(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, c, a, i);
    nnml_compute_forward_set_rows(node, &s.st);
    memcpy(cache, node->tensor_data(), (size_t)n_cells * n * 2);
}

// ADD (binary.cpp) of two [n] fp32 vectors
void ref_add_f32(const float * a, const float * b, float * y, int64_t n) {
    auto mem = make_mem((size_t)n * 4 * 4 + (1 << 20));
    state s;
    nnml_tensor * ta = nnml_tensor::new_1d(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, NNML_TYPE_F32, n);
    nnml_tensor * tb = nnml_tensor::new_1d(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, NNML_TYPE_F32, n);
    memcpy(ta->tensor_data(), a, (size_t)n * 4);
    memcpy(tb->tensor_data(), b, (size_t)n * 4);
    nnml_tensor * node = nnml_add(mem, NNML_TENSOR_TYPE_ACTIVATION, 0, 0, ta, tb);
    nnml_compute_forward_add(node, &s.st);
    memcpy(y, node->tensor_data(), (size_t)n * 4);
}

}  // extern "C"
