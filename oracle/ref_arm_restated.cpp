// Portable restatement of the NEON-only nnml symbols that the reference's
// portable sources reference (nnml/src/ops/arm/arm.cpp, gemm.cpp).  Linked only
// into oracle/_ref/libalref.so so that the reference's own ops.cpp / types.cpp /
// binary.cpp / common.cpp / tensor.cpp / memory.cpp can be loaded on x86.
// Test infrastructure only.  Functions the golden-vector driver never reaches
// abort loudly instead of guessing.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "ops.h"
#include "tensor.h"

static inline float h2f(nnml_fp16_t h) { return nnml_compute_fp16_to_fp32(h); }

[[noreturn]] static void not_restated(const char * fn) {
    fprintf(stderr, "oracle/_ref: %s is not restated for the x86 reference build\n", fn);
    abort();
}

// arm.cpp:169-179
void nnml_cpu_fp16_to_fp32(const nnml_fp16_t * x, float * y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = h2f(x[i]);
}
float f16_to_f32(nnml_fp16_t x) { return h2f(x); }

// arm.cpp:1453-1500 (y *= v)
void nnml_vec_scale_f32(const int n, float * y, const float v) {
    for (int i = 0; i < n; ++i) y[i] *= v;
}

// arm.cpp:1789-1809 (silu(x) * g, libm expf)
void nnml_vec_swiglu_f32(const int n, float * y, const float * x, const float * g) {
    for (int i = 0; i < n; ++i) y[i] = (x[i] / (1.0f + expf(-x[i]))) * g[i];
}

// arm.cpp:2435-2477
void nnml_vec_add_f32(float * dst, const float ** srcs, int n_srcs, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float s = srcs[0][i];
        for (int j = 1; j < n_srcs; ++j) s += srcs[j][i];
        dst[i] = s;
    }
}
void nnml_vec_add_f16(_Float16 * dst, const _Float16 ** srcs, int n_srcs, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        _Float16 s = srcs[0][i];
        for (int j = 1; j < n_srcs; ++j) s = (_Float16)((double)s + (double)srcs[j][i]);
        dst[i] = s;
    }
}

// arm.cpp:1819-1853 (round to nearest even)
void quantize_row_q8_0(const float * x, void * vy, int64_t k) {
    block_q8_0 * y = (block_q8_0 *)vy;
    const int nb = (int)(k / QK8_0);
    for (int i = 0; i < nb; i++) {
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; j++) amax = std::fmax(amax, std::fabs(x[i * QK8_0 + j]));
        const float d = amax / ((1 << 7) - 1);
        const float id = d ? 1.0f / d : 0.0f;
        y[i].d = nnml_compute_fp32_to_fp16(d);
        for (int j = 0; j < QK8_0; ++j) y[i].qs[j] = (int8_t)std::nearbyint(x[i * QK8_0 + j] * id);
    }
}

// arm.cpp:675-691 scalar semantics
void nnml_vec_dot_q4_0_q8_0(int n, float * s, size_t, const void * vx, size_t, const void * vy, size_t, int) {
    const block_q4_0 * x = (const block_q4_0 *)vx;
    const block_q8_0 * y = (const block_q8_0 *)vy;
    float sumf = 0.0f;
    for (int ib = 0; ib < n / QK8_0; ++ib) {
        int sumi = 0;
        for (int j = 0; j < QK8_0 / 2; ++j) {
            sumi += ((x[ib].qs[j] & 0x0F) - 8) * y[ib].qs[j];
            sumi += ((x[ib].qs[j] >> 4) - 8) * y[ib].qs[j + QK8_0 / 2];
        }
        sumf += sumi * h2f(x[ib].d) * h2f(y[ib].d);
    }
    *s = sumf;
}

void nnml_vec_dot_f32(int, float *, size_t, const float *, size_t, const float *, size_t, int) { not_restated(__func__); }
void nnml_vec_dot_f16(int, float *, size_t, nnml_fp16_t *, size_t, nnml_fp16_t *, size_t, int) { not_restated(__func__); }
void nnml_vec_dot_q8_0_q8_0(int, float *, size_t, const void *, size_t, const void *, size_t, int) { not_restated(__func__); }
void nnml_vec_dot_q6_K_q8_K(int, float *, size_t, const void *, size_t, const void *, size_t, int) { not_restated(__func__); }
void nnml_compute_forward_flash_attn_ext_f16(nnml_tensor *, const nnml_compute_state *) { not_restated(__func__); }
void nnml_compute_forward_rope_f16(nnml_tensor *, const nnml_compute_state *) { not_restated(__func__); }
void nnml_compute_forward_soft_max_f32(nnml_tensor *, const nnml_compute_state *) { not_restated(__func__); }

// thread.cpp: single-threaded driver, so the global barrier is a no-op.
void nnml_barrier_global(nnml_threadpool *) {}
int nnml_get_boot_node_id() { return 0; }
