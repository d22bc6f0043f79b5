/* nnml_gpu_ops: the reference's operators for the Qwen3 decode path as GPU
 * operators over libalb_cuda.so, in the shape nnml calls them.
 *
 * nnml runs every operator from every pool thread as f(params, node) and each
 * thread takes a slice by ith / nth (ops.h:414-433, arm.cpp:1862-1909); on the
 * GPU the whole operator is one stream-ordered launch by thread 0 of the group,
 * the others return.  The tensor view keeps the fields the operators read
 * (tensor.h:98-183: ne, nb, data, op_params, src); `data` is device memory.
 * The state carries the GPU context's stream and DEVICE scratch: nnml's own
 * params->work_data is host memory (thread.h:166-167) and is never handed to a
 * kernel.  Every function returns an alb status (ALB_OK = 0); the reference
 * aborts instead (nnml.h:97-111). */
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "alb_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct nnml_gpu_tensor {
    int64_t ne[4];                          /* elements per dimension, ne[0] innermost */
    size_t nb[4];                           /* byte strides */
    void * data;                            /* device memory */
    int32_t op_params[16];
    const struct nnml_gpu_tensor * src[4];
} nnml_gpu_tensor;

typedef struct nnml_gpu_state {
    int32_t ith, nth;                       /* pool thread and group size (only ith == 0 launches) */
    void * stream;                          /* the context's cudaStream_t */
    void * xq;  size_t xq_bytes;            /* device scratch: a mat-vec's block_q8_0 input */
    void * attn_ws; size_t attn_ws_bytes;   /* device scratch: alb_flash_attn workspace */
} nnml_gpu_state;

/* MUL_MAT, one activation row (ne11 == 1): dst [N] = src0 (Q4_0, alb GPU
 * layout, [N][K]) x src1 (fp32 [K]).  op_params[0] = 1: the weight is one the
 * reference repacks to 4x4 (nnml_gemv_q4_0_4x4_q8_0 chain, gemm.cpp:127-190);
 * 0: a plain Q4_0 weight (vec_dot_q4_0_q8_0 chain, arm.cpp:633-692, the output
 * matrix, model.cpp:342-353). */
ALB_API int nnml_gpu_forward_mul_mat(const nnml_gpu_state * params, nnml_gpu_tensor * dst);
/* RMS_NORM then the graph's MUL (ops.cpp:680-724, binary.cpp:15-23): dst [rows][n] =
 * rms_norm(src0) * src1 [n]; op_params[0] = eps (float bits). */
ALB_API int nnml_gpu_forward_rms_norm_mul(const nnml_gpu_state * params, nnml_gpu_tensor * dst);
/* GET_ROWS of a Q4_0 table (ops.cpp:12-52): dst [n_ids][K] fp32, src0 table
 * (alb GPU layout [n_rows][K]), src1 int32 ids [n_ids]. */
ALB_API int nnml_gpu_forward_get_rows(const nnml_gpu_state * params, nnml_gpu_tensor * dst);
/* SET_ROWS into an fp16 array (ops.cpp:135-181, the KV store of cpy_k / cpy_v,
 * cgraph.cpp:1114-1180): dst fp16 [rows][row_len] (the cache view) gets row
 * src1[r] := fp16(src0 row r) for the fp32 rows src0 [n][row_len] and the int64
 * indices src1 [n] (device; e.g. alb_kv_prepare's cells). */
ALB_API int nnml_gpu_forward_set_rows(const nnml_gpu_state * params, nnml_gpu_tensor * dst);
/* GLU/SWIGLU, split form (ops.cpp:1038-1092): dst [n] = silu(src0) * src1. */
ALB_API int nnml_gpu_forward_swiglu(const nnml_gpu_state * params, nnml_gpu_tensor * dst);
/* FLASH_ATTN_EXT (arm.cpp:2196-2433), one sequence, causal: dst and src0 (q)
 * [T][n_head][128] fp32, src1 / src2 the fp16 K / V caches [cells][n_head_kv][128];
 * op_params[0] = pos0 (token t at position pos0 + t), [1] = scale (float bits),
 * [2] = splits. */
ALB_API int nnml_gpu_forward_flash_attn_ext(const nnml_gpu_state * params, nnml_gpu_tensor * dst);
/* sample_none (sampler.cpp:34-36): dst int32 [1] (device) = first index of the
 * maximum of src0 fp32 [n]; uses params->attn_ws (>= 1024 bytes, zeroed once) as
 * the argmax scratch. */
ALB_API int nnml_gpu_sample_greedy(const nnml_gpu_state * params, nnml_gpu_tensor * dst);

#ifdef __cplusplus
}
#endif
