// Internal (C++) interface between the C ABI, the kernels and the Qwen3 engine.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "alb_cuda.h"

namespace alb {

// How a GEMV obtains its Q8_0 activation vector.
enum GemvIn : int {
    GEMV_IN_Q8 = 0,       // block_q8_0 [K/32] in global memory (reference layout)
    GEMV_IN_F32 = 1,      // fp32 [K]: quantized to Q8_0 in the prologue (arm.cpp:1886-1897)
    GEMV_IN_F32_RMS = 2,  // fp32 [K]: RMSNorm (ops.cpp:680-724) * w, then quantized
};

// What a GEMV writes, and which of the reference's summation chains it runs.
// PLAIN / SWIGLU / DOTS: nnml_gemv_q4_0_4x4_q8_0 (gemm.cpp:127-190), one fp32
// fma chain per row over its blocks in order.  PAIR / LOGITS: the generic
// mul_mat's nnml_vec_dot_q4_0_q8_0 (arm.cpp:633-692): eight lane chains
// (block parity x 4 partial dots) then a fixed add tree.
enum GemvOut : int {
    GEMV_OUT_PLAIN = 0,   // y[n] = acc (+ residual[n])
    GEMV_OUT_SWIGLU = 1,  // rows interleaved (gate n, up n): y[n] = silu(gate)*up (ops.cpp:1038-1092)
    GEMV_OUT_DOTS = 2,    // y[n] = acc and I[n][b] = int32 block dots (parity check)
    GEMV_OUT_PAIR = 3,    // y[n] = vec_dot(W[n], x)
    GEMV_OUT_LOGITS = 4,  // PAIR, plus the greedy argmax key (and, with `next`, the token)
};

struct GemvArgs {
    const uint8_t * W = nullptr;   // row 0 of this view of the alb Q4_0 GPU layout (16-byte aligned)
    int64_t N = 0, K = 0;          // physical rows, columns
    int in_mode = GEMV_IN_Q8;
    const void * x = nullptr;      // block_q8_0 or fp32 per in_mode
    const float * norm_w = nullptr;
    float eps = 1e-6f;
    int out_mode = GEMV_OUT_PLAIN;
    float * y = nullptr;
    const float * residual = nullptr;
    int32_t * dots = nullptr;
    bool pdl = false;              // launch as a programmatic dependent
    int ctas = 0;                  // grid size (0 = one CTA per SM)
    int smem_budget = 0;           // bytes of dynamic shared memory (0 = default)
    int * err = nullptr;           // device error word (filled by launch_gemv)
    // LOGITS only: running argmax key (ordered value << 32 | ~index; zeroed
    // before the launch), row index offset of this shard, and optionally the
    // token output: the last CTA (ticket, zero before the first launch, re-armed)
    // turns the key into the index
    unsigned long long * key = nullptr;
    int64_t idx_base = 0;
    int * ticket = nullptr;
    int32_t * next = nullptr;
};

struct FlashArgs {
    const float * q = nullptr;          // [T][Hq][128] fp32
    const uint16_t * kc = nullptr;      // [cells][Hkv][128] fp16
    const uint16_t * vc = nullptr;
    int Hq = 0, Hkv = 0, T = 1;
    int32_t pos0 = 0;                   // position of token 0 (ignored when pos_dev)
    const int32_t * pos_dev = nullptr;  // device-resident pos0 (CUDA-graph replay)
    float scale = 0.0f;
    int S = 1;                          // splits along the cells
    int ncap = 0;                       // upper bound of cells attended (>= pos0 + T)
    float * ws = nullptr;               // flash_attn_ws_bytes()
    float * out = nullptr;              // [T][Hq][128] fp32
    void * xq = nullptr;                // optional: block_q8_0 records of out, [T][Hq*4]
    float * sws = nullptr;              // optional, prefill: score workspace (fa_prefill_scores_bytes)
    bool pdl = false;
};
// Bytes of the prefill attention's score workspace for T tokens over ncap cells.
size_t fa_prefill_scores_bytes(int Hq, int Hkv, int T, int ncap);
size_t flash_attn_ws_bytes(int Hq, int Hkv, int T, int S, int ncap);
size_t split_attn_ws_bytes(int Hq, int Hkv, int T, int S, int ncap);
cudaError_t launch_split_attn(const FlashArgs & f, cudaStream_t st);
// false when the call's kernels need no workspace (launch_flash_attn's path choice)
bool flash_attn_uses_ws(int Hq, int Hkv, int T, int S, int ncap);
cudaError_t launch_flash_attn(const FlashArgs & f, cudaStream_t st);

struct QkvArgs {
    const float * qkv = nullptr;        // [T][qkv_stride]: q (Hq*128) | k (Hkv*128) | v (Hkv*128)
    int64_t qkv_stride = 0;
    int Hq = 0, Hkv = 0, T = 1;
    const float * q_norm = nullptr, * k_norm = nullptr;
    float eps = 1e-6f;
    const float2 * rope = nullptr;      // [max_pos][64] (cos, sin)
    int32_t pos0 = 0;
    const int32_t * pos_dev = nullptr;
    float * q_out = nullptr;            // [T][Hq][128]
    uint16_t * kc = nullptr, * vc = nullptr;  // cache base of this layer [cells][Hkv][128]
    bool pdl = false;
    // optional, device, per token: positions and cells (else pos0 + t for both)
    const int32_t * pos_tok = nullptr;
    const int64_t * cell_tok = nullptr;
    int64_t n_cells = 0;                // cache rows (bound of cell_tok)
    int32_t max_pos = 0;                // RoPE table rows (bound of pos_tok)
};
cudaError_t launch_qk_norm_rope_kv(const QkvArgs & a, cudaStream_t st);
// Decode step attention with QK-norm + RoPE + the K/V store fused (T = 1):
// f describes the attention (workspace, splits, output and its Q8_0 records),
// qa the raw QKV projection, norm weights, RoPE table and the caches to store into.
// Decode-step attention of one token from the raw QKV projection (QK-norm,
// RoPE and the new K/V cell included): one cluster launch when `cluster`
// (f.ncap <= attn_decode_cluster_max_cells()), else the two split kernels.
cudaError_t launch_attn_decode(const FlashArgs & f, const QkvArgs & qa, bool cluster, cudaStream_t st);
int attn_decode_cluster_max_cells();
cudaError_t launch_embed(const uint8_t * W, int64_t vocab, int64_t E, const int32_t * tokens, int T, float * x,
                         unsigned long long * key_reset, bool pdl, cudaStream_t st);
// argmax over x[0..n): scratch >= 64*8 + 16 bytes with its ticket word zero at first use
cudaError_t launch_argmax(const float * x, int64_t n, int64_t idx_base, void * scratch,
                          unsigned long long * key_out, int32_t * idx_out, bool pdl, cudaStream_t st);
cudaError_t launch_key_to_index(const unsigned long long * key, int32_t * idx, bool pdl, cudaStream_t st);
cudaError_t launch_rms_norm(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps, bool pdl,
                            cudaStream_t st);
// RMSNorm (+ MUL by w) / swiglu followed by quantize_row_q8_0 of the result;
// y (fp32 copy of the result) may be null; n % 32 == 0.
cudaError_t launch_rms_norm_q8(const float * x, const float * w, float * y, void * yq, int64_t rows, int64_t n,
                               float eps, bool pdl, cudaStream_t st);
// quantize_row_q8_0 of n fp32 values (n % 32 == 0) -> block_q8_0 [n/32]
cudaError_t launch_quantize_q8_0(const float * x, void * xq, int64_t n, bool pdl, cudaStream_t st);
cudaError_t launch_swiglu_q8(const float * g, const float * u, float * y, void * yq, int64_t n, bool pdl,
                             cudaStream_t st);
cudaError_t launch_swiglu(const float * g, const float * u, float * y, int64_t n, bool pdl, cudaStream_t st);
cudaError_t launch_set_rows_f16(const float * src, int64_t n_rows, int64_t row_len, const int64_t * idx, uint16_t * dst,
                                int64_t dst_rows, cudaStream_t st);
cudaError_t launch_get_rows_f16(const uint16_t * src, int64_t src_rows, int64_t row_len, const int64_t * idx,
                                int64_t n_rows, uint16_t * dst, cudaStream_t st);

// Sets a kernel's dynamic shared-memory limit on the current device when
// `bytes` exceeds what was set there before (thread safe, per device).
cudaError_t ensure_dynamic_smem(const void * func, size_t bytes);
template <typename F> inline cudaError_t ensure_smem(F * func, size_t bytes) {
    return ensure_dynamic_smem(reinterpret_cast<const void *>(func), bytes);
}

// Device-side error word (bounded waits that expire set it; see alb_device_error).
enum : int { ALB_DEVERR_NONE = 0, ALB_DEVERR_MBAR_TIMEOUT = 1, ALB_DEVERR_FLAG_TIMEOUT = 2, ALB_DEVERR_BAD_TOKEN = 3,
             ALB_DEVERR_BAD_INDEX = 4 };
// Host: the current device's error word (allocated once per device, zeroed).
int * device_error_ptr();

cudaError_t launch_gemv(const GemvArgs & a, cudaStream_t stream);
// prefill mat-mul on the tensor cores: x fp32 [M][K] (or, x == nullptr, block_q8_0
// rows xq_blocks) times W [N][K] -> y [M][y_stride] (SwiGLU: y [M][N/2]);
// workspace prefill_ws_bytes(M, K)
size_t prefill_ws_bytes(int64_t M, int64_t K);
cudaError_t launch_prefill_gemm(const uint8_t * W, int64_t N, int64_t K, const float * x, const void * xq_blocks,
                                int64_t M, float * y, int64_t y_stride, const float * residual, bool swiglu, void * ws,
                                int * err, bool pdl, cudaStream_t st);

// alb Q4_0 GPU layout, row-interleaved: row n occupies q4_row_bytes(K) bytes at
// n * q4_row_bytes(K): the K/2 nibble bytes (block b's 16 qs bytes at 16 b),
// then the K/32 fp16 scales padded with zeros to q4_scale_pitch(K) entries (a
// 16-byte multiple).  Any run of consecutive rows is one contiguous, 16-byte
// aligned range: one bulk copy brings a whole stage of rows.
__host__ __device__ inline int64_t q4_scale_pitch(int64_t K) {   // in fp16 elements
    return ((K / 32) + 7) & ~(int64_t)7;
}
__host__ __device__ inline int64_t q4_row_bytes(int64_t K) {
    return K / 2 + q4_scale_pitch(K) * 2;
}
__host__ __device__ inline size_t q4_gpu_bytes(int64_t N, int64_t K) {
    return ((size_t)N * (size_t)q4_row_bytes(K) + 255) & ~(size_t)255;
}

}  // namespace alb
