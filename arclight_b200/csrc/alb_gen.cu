// Seeded synthetic Qwen3 weights, generated directly on the device in the alb
// Q4_0 GPU layout.  The stream is defined (identically in the oracle) as
//   z(seed, idx) = inverse-normal-CDF table lookup with linear interpolation,
//   table[j] = Acklam's rational approximation at (j + 0.5) / 65537,
//   index from splitmix64(seed + idx * 0xD1B54A32D192ED03);
//   W[r][c] = 0.02 * z(seed_W, r * K + c) quantized with quantize_row_q4_0_ref
//   (types.cpp:352-378); norm weights = 1 + 0.01 * z(seed_w, i).
// Every element is indexed by its position in the FULL tensor, so a tensor
// parallel shard generates exactly the rows / columns of the unsharded model.
#include <cmath>
#include <vector>

#include "alb_common.cuh"
#include "alb_internal.h"

namespace alb {

uint64_t splitmix64_host(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

uint64_t tensor_seed(uint64_t model_seed, int layer, int kind) {
    return splitmix64_host(model_seed * 0x100000001B3ULL + (uint64_t)((layer + 1) * 64 + kind));
}

// P. J. Acklam's inverse normal CDF approximation (double), table definition.
static double inv_norm(double p) {
    static const double a[6] = {-3.969683028665376e+01, 2.209460984245205e+02, -2.759285104469687e+02,
                                1.383577518672690e+02, -3.066479806614716e+01, 2.506628277459239e+00};
    static const double b[5] = {-5.447609879822406e+01, 1.615858368580409e+02, -1.556989798598866e+02,
                                6.680131188771972e+01, -1.328068155288572e+01};
    static const double c[6] = {-7.784894002430293e-03, -3.223964580411365e-01, -2.400758277161838e+00,
                                -2.549732539343734e+00, 4.374664141464968e+00, 2.938163982698783e+00};
    static const double d[4] = {7.784695709041462e-03, 3.224671290700398e-01, 2.445134137142996e+00,
                                3.754408661907416e+00};
    const double plow = 0.02425, phigh = 1.0 - plow;
    if (p < plow) {
        const double q = sqrt(-2.0 * log(p));
        return (((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
               ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1.0);
    }
    if (p <= phigh) {
        const double q = p - 0.5, r = q * q;
        return (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q /
               (((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1.0);
    }
    const double q = sqrt(-2.0 * log(1.0 - p));
    return -(((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
           ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1.0);
}

void normal_table_host(std::vector<float> & t) {
    t.resize(65537);
    for (int j = 0; j <= 65536; ++j) t[j] = (float)inv_norm(((double)j + 0.5) / 65537.0);
}

__device__ __forceinline__ uint64_t d_splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float d_normal(const float * __restrict__ t, uint64_t seed, uint64_t idx) {
    const uint64_t h = d_splitmix64(seed + idx * 0xD1B54A32D192ED03ULL);
    const uint32_t i = (uint32_t)(h >> 48);
    const float frac = __fmul_rn((float)((h >> 24) & 0xFFFFFFu), 1.0f / 16777216.0f);
    const float lo = t[i], hi = t[i + 1];
    return __fmaf_rn(frac, __fsub_rn(hi, lo), lo);
}

// One thread per (row, block).  quantize_row_q4_0_ref: first max-abs element,
// d = max / -8, id = 1/d, q = min(15, (int8)(x*id + 8.5)), d stored fp16.
__global__ void k_gen_q4(uint8_t * __restrict__ W, int64_t K, int64_t sp,
                         int64_t dst_row0, int64_t dst_row_stride, int64_t n_rows, uint64_t seed,
                         int64_t src_row0, int64_t K_full, int64_t c0, const float * __restrict__ table, float stdv) {
    const int64_t nb = K / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_rows * nb) return;
    const int64_t r = i / nb, b = i - r * nb;
    const uint64_t base = (uint64_t)(src_row0 + r) * (uint64_t)K_full + (uint64_t)(c0 + 32 * b);
    float v[32];
    float amax = 0.0f, mx = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        v[j] = __fmul_rn(stdv, d_normal(table, seed, base + j));
        if (amax < fabsf(v[j])) { amax = fabsf(v[j]); mx = v[j]; }
    }
    const float d = __fdiv_rn(mx, -8.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    uint32_t words[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int t0 = (int)(int8_t)__float2int_rz(__fadd_rn(__fmul_rn(v[j], id), 8.5f));
        const int t1 = (int)(int8_t)__float2int_rz(__fadd_rn(__fmul_rn(v[j + 16], id), 8.5f));
        const uint32_t q0 = (uint32_t)(t0 < 15 ? t0 : 15) & 0xFF, q1 = (uint32_t)(t1 < 15 ? t1 : 15) & 0xFF;
        words[j >> 2] |= ((q0 | (q1 << 4)) & 0xFF) << (8 * (j & 3));
    }
    const int64_t drow = dst_row0 + r * dst_row_stride;
    uint8_t * row = W + drow * q4_row_bytes(K);   // row-interleaved GPU layout
    *reinterpret_cast<uint4 *>(row + 16 * b) = make_uint4(words[0], words[1], words[2], words[3]);
    uint16_t * srow = reinterpret_cast<uint16_t *>(row + K / 2);
    srow[b] = alb_f2h(d);
    if (b == nb - 1)
        for (int64_t j = nb; j < sp; ++j) srow[j] = 0;
}

__global__ void k_gen_norm(float * __restrict__ w, int64_t n, uint64_t seed, const float * __restrict__ table) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) w[i] = __fadd_rn(1.0f, __fmul_rn(0.01f, d_normal(table, seed, (uint64_t)i)));
}

// fp16 values ~ N(0, 1) (config 5 KV pre-fill): cache [cells][row] of one shard;
// element (cell, c) of the shard is element (cell, col0 + c) of the full row.
__global__ void k_gen_f16(uint16_t * __restrict__ dst, int64_t cells, int64_t row, int64_t full_row, int64_t col0,
                          uint64_t seed, const float * __restrict__ table) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= cells * row) return;
    const int64_t c = i / row, e = i - c * row;
    dst[i] = alb_f2h(d_normal(table, seed, (uint64_t)c * full_row + col0 + e));
}

cudaError_t gen_q4(uint8_t * W, int64_t N_total, int64_t K, int64_t dst_row0, int64_t dst_row_stride, int64_t n_rows,
                   uint64_t seed, int64_t src_row0, int64_t K_full, int64_t c0, const float * table, cudaStream_t st) {
    const int64_t n = n_rows * (K / 32);
    (void)N_total;
    k_gen_q4<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(W, K, q4_scale_pitch(K), dst_row0, dst_row_stride, n_rows,
                                                         seed, src_row0, K_full, c0, table, 0.02f);
    return cudaGetLastError();
}

cudaError_t gen_norm(float * w, int64_t n, uint64_t seed, const float * table, cudaStream_t st) {
    k_gen_norm<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w, n, seed, table);
    return cudaGetLastError();
}

cudaError_t gen_f16(uint16_t * dst, int64_t cells, int64_t row, int64_t full_row, int64_t col0, uint64_t seed,
                    const float * table, cudaStream_t st) {
    const int64_t n = cells * row;
    k_gen_f16<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(dst, cells, row, full_row, col0, seed, table);
    return cudaGetLastError();
}

}  // namespace alb
