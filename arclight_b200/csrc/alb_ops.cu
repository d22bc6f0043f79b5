// Elementwise / attention / sampling kernels of the Qwen3 decode/prefill path
// (sm_100a).  Reference semantics cited per kernel.
#include <cfloat>
#include <cmath>

#include "alb_common.cuh"
#include "alb_internal.h"

namespace alb {

// ------------------------------------------------------------------ embedding
// GET_ROWS on the Q4_0 token table (ops.cpp:12-52, dequantize_row_q4_0
// types.cpp:337-350): x[t][j] = (q - 8) * d.  One thread per 32-value block.
__global__ void k_embed_q4_0(const uint8_t * __restrict__ Wn, const uint16_t * __restrict__ Ws, int64_t sp,
                             const int32_t * __restrict__ tokens, int T, int64_t E, int64_t vocab,
                             float * __restrict__ x, int * err) {
    const int64_t nb = E / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * nb) return;
    const int t = (int)(i / nb), b = (int)(i - (int64_t)t * nb);
    alb_pdl_wait();
    int32_t tok = tokens[t];
    if (tok < 0 || tok >= vocab) { atomicExch(err, 3); tok = 0; }
    const uint4 v = *reinterpret_cast<const uint4 *>(Wn + (size_t)tok * (E / 2) + 16 * b);
    const float d = alb_h2f(Ws[(size_t)tok * sp + b]);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float * o = x + (size_t)t * E + 32 * b;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int byte = (w[k] >> (8 * j)) & 0xFF;
            o[4 * k + j] = (float)((byte & 0x0F) - 8) * d;
            o[16 + 4 * k + j] = (float)((byte >> 4) - 8) * d;
        }
    alb_pdl_trigger();
}

// ------------------------------------------------- QK-norm + RoPE + KV store
// Per token t and head: Q heads get RMSNorm(128)*q_norm (qwen3.cpp:215-217,
// ops.cpp:680-724) then NEOX RoPE at pos0+t (ops.cpp:830-938) using the host
// cos/sin table (nnml_rope_cache_init, ops.cpp:759-771); K heads likewise with
// k_norm and are stored fp32->fp16 (RNE) into the K cache row pos0+t
// (set_rows, ops.cpp:135-181); V heads are stored as is.
// Block = 128 threads (one per dimension), grid = (Hq + 2*Hkv, T).
__global__ void __launch_bounds__(128)
k_qk_norm_rope_kv(const float * __restrict__ qkv, int64_t qkv_stride, int Hq, int Hkv,
                  const float * __restrict__ qn_w, const float * __restrict__ kn_w, float eps,
                  const float2 * __restrict__ rope, int32_t pos0, const int32_t * __restrict__ pos_dev,
                  float * __restrict__ q_out, uint16_t * __restrict__ kc, uint16_t * __restrict__ vc,
                  int64_t kv_row) {
    const int head = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
    const int lane = d & 31, warp = d >> 5;
    alb_pdl_wait();
    const int32_t pos = (pos_dev ? pos_dev[0] : pos0) + t;
    const float * src = qkv + (size_t)t * qkv_stride;
    __shared__ float buf[128];
    __shared__ double red[4];
    if (head >= Hq + Hkv) {   // V head: plain fp16 store
        const int hv = head - Hq - Hkv;
        vc[(size_t)pos * kv_row + hv * 128 + d] = alb_f2h(src[(Hq + Hkv) * 128 + hv * 128 + d]);
        alb_pdl_trigger();
        return;
    }
    const bool is_q = head < Hq;
    const int hh = is_q ? head : head - Hq;
    const float v = src[(is_q ? 0 : Hq * 128) + hh * 128 + d];
    double s = (double)__fmul_rn(v, v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    // reference order: ((s0 + s1) + s2) + s3 over 32-lane partials of a sequential
    // double sum -- any order of 128 fp32 squares in double rounds identically
    const double tot = red[0] + red[1] + red[2] + red[3];
    const float mean = (float)(tot / 128.0);
    const float scale = 1.0f / sqrtf(__fadd_rn(mean, eps));
    const float nv = __fmul_rn(__fmul_rn(v, scale), (is_q ? qn_w : kn_w)[d]);
    buf[d] = nv;
    __syncthreads();
    float outv;
    const float2 cs = rope[(size_t)pos * 64 + (d & 63)];
    if (d < 64) outv = __fsub_rn(__fmul_rn(buf[d], cs.x), __fmul_rn(buf[d + 64], cs.y));
    else        outv = __fadd_rn(__fmul_rn(buf[d - 64], cs.y), __fmul_rn(buf[d], cs.x));
    if (is_q) q_out[((size_t)t * Hq + hh) * 128 + d] = outv;
    else      kc[(size_t)pos * kv_row + hh * 128 + d] = alb_f2h(outv);
    alb_pdl_trigger();
}

// ------------------------------------------------------------ flash attention
// nnml_compute_forward_flash_attn_ext_f16 (arm.cpp:2196-2433) for F16 K/V,
// one sequence, causal: token t (position p0 + t) attends cells [0, p0+t+1).
// Q is rounded to fp16 first as the reference does (arm.cpp:2307); scores,
// softmax and the V accumulation are fp32 (the reference accumulates V in
// fp16; fp32 is the more accurate choice and stays well inside 1e-3).
// Split-K over the cells: CTA (kv head h, token t, split s) runs an online
// softmax over its cell range for the G = Hq/Hkv query heads of h and writes
// (m, l, acc) to the workspace; the last CTA of (h, t) (atomic ticket, no
// spin) merges the splits with the usual log-sum-exp rescale.
template <int G>
__global__ void __launch_bounds__(128)
k_flash_attn(const float * __restrict__ q, const uint16_t * __restrict__ kc, const uint16_t * __restrict__ vc,
             int Hq, int Hkv, int T, int32_t pos0, const int32_t * __restrict__ pos_dev, float scale,
             int S, float * __restrict__ ws, int * __restrict__ tickets, float * __restrict__ out) {
    const int h = blockIdx.x, t = blockIdx.y, s = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int D = 128;
    __shared__ float qs[G][D];
    __shared__ float wm[4][G], wl[4][G];
    __shared__ float wacc[4][G][D];
    __shared__ int last;
    alb_pdl_wait();
    const int32_t p0 = pos_dev ? pos_dev[0] : pos0;
    const int n = p0 + t + 1;
    const int64_t row = (int64_t)Hkv * D;
    for (int i = tid; i < G * D; i += 128) {
        const int g = i / D, d = i - g * D;
        qs[g][d] = __half2float(__float2half_rn(q[((size_t)t * Hq + h * G + g) * D + d]));
    }
    __syncthreads();
    int sz = (n + S - 1) / S;
    sz = (sz + 31) & ~31;
    const int c0 = s * sz, c1 = min(n, c0 + sz);

    float m[G], l[G], acc[G][4];
#pragma unroll
    for (int g = 0; g < G; ++g) { m[g] = -INFINITY; l[g] = 0.0f; acc[g][0] = acc[g][1] = acc[g][2] = acc[g][3] = 0.0f; }

    for (int base = c0 + warp * 32; base < c1; base += 128) {
        const int c = base + lane;
        float sc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) sc[g] = -INFINITY;
        if (c < c1) {
            const uint4 * kr = reinterpret_cast<const uint4 *>(kc + (size_t)c * row + (size_t)h * D);
            float a[G];
#pragma unroll
            for (int g = 0; g < G; ++g) a[g] = 0.0f;
#pragma unroll 4
            for (int j = 0; j < 16; ++j) {
                const uint4 kv = kr[j];
                const uint32_t wd[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 kf = __half22float2(*reinterpret_cast<const __half2 *>(&wd[e]));
                    const int d = 8 * j + 2 * e;
#pragma unroll
                    for (int g = 0; g < G; ++g) a[g] = fmaf(kf.y, qs[g][d + 1], fmaf(kf.x, qs[g][d], a[g]));
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) sc[g] = a[g] * scale;
        }
        float p[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float cm = alb_warp_max(sc[g]);
            const float mn = fmaxf(m[g], cm);
            const float r = (m[g] == -INFINITY) ? 0.0f : expf(m[g] - mn);
            p[g] = (c < c1) ? expf(sc[g] - mn) : 0.0f;
            l[g] = l[g] * r + alb_warp_sum(p[g]);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[g][e] *= r;
            m[g] = mn;
        }
        const int nc = min(32, c1 - base);
        for (int j = 0; j < nc; ++j) {
            const uint2 vv = *reinterpret_cast<const uint2 *>(vc + (size_t)(base + j) * row + (size_t)h * D + 4 * lane);
            const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.x));
            const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.y));
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float pj = __shfl_sync(0xffffffffu, p[g], j);
                acc[g][0] = fmaf(v01.x, pj, acc[g][0]);
                acc[g][1] = fmaf(v01.y, pj, acc[g][1]);
                acc[g][2] = fmaf(v23.x, pj, acc[g][2]);
                acc[g][3] = fmaf(v23.y, pj, acc[g][3]);
            }
        }
    }
    // merge the 4 warps of this CTA
    if (lane == 0)
#pragma unroll
        for (int g = 0; g < G; ++g) { wm[warp][g] = m[g]; wl[warp][g] = l[g]; }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < 4; ++e) wacc[warp][g][4 * lane + e] = acc[g][e];
    __syncthreads();
    // thread tid owns dimension tid for every head
    float M[G], Lsum[G], O[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float mx = -INFINITY;
        for (int w = 0; w < 4; ++w) mx = fmaxf(mx, wm[w][g]);
        float L = 0.0f, o = 0.0f;
        for (int w = 0; w < 4; ++w) {
            const float f = (wm[w][g] == -INFINITY) ? 0.0f : expf(wm[w][g] - mx);
            L += wl[w][g] * f;
            o += wacc[w][g][tid] * f;
        }
        M[g] = mx; Lsum[g] = L; O[g] = o;
    }
    if (S == 1) {
#pragma unroll
        for (int g = 0; g < G; ++g)
            out[((size_t)t * Hq + h * G + g) * D + tid] = Lsum[g] > 0.0f ? O[g] / Lsum[g] : 0.0f;
        alb_pdl_trigger();
        return;
    }
    // write the split partial: [h][t][s][G][D + 2]
    float * part = ws + (((size_t)h * T + t) * S + s) * G * (D + 2);
#pragma unroll
    for (int g = 0; g < G; ++g) {
        part[g * (D + 2) + tid] = O[g];
        if (tid == 0) { part[g * (D + 2) + D] = M[g]; part[g * (D + 2) + D + 1] = Lsum[g]; }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = (atomicAdd(&tickets[h * T + t], 1) == S - 1);
    __syncthreads();
    if (!last) { alb_pdl_trigger(); return; }
    __threadfence();
    const float * base = ws + ((size_t)h * T + t) * S * G * (D + 2);
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float mx = -INFINITY;
        for (int k = 0; k < S; ++k) mx = fmaxf(mx, __ldcg(base + ((size_t)k * G + g) * (D + 2) + D));
        float L = 0.0f, o = 0.0f;
        for (int k = 0; k < S; ++k) {
            const float * pk = base + ((size_t)k * G + g) * (D + 2);
            const float mk = __ldcg(pk + D);
            const float f = (mk == -INFINITY) ? 0.0f : expf(mk - mx);
            L += __ldcg(pk + D + 1) * f;
            o += __ldcg(pk + tid) * f;
        }
        out[((size_t)t * Hq + h * G + g) * D + tid] = L > 0.0f ? o / L : 0.0f;
    }
    if (tid == 0) tickets[h * T + t] = 0;   // re-arm for the next launch / graph replay
    alb_pdl_trigger();
}

size_t flash_attn_ws_bytes(int Hq, int Hkv, int T, int S) {
    const int G = Hq / Hkv;
    return (size_t)Hkv * T * S * G * (128 + 2) * 4 + (size_t)Hkv * T * 4 + 256;
}

cudaError_t launch_flash_attn(const FlashArgs & f, cudaStream_t st) {
    const int G = f.Hq / f.Hkv;
    dim3 grid((unsigned)f.Hkv, (unsigned)f.T, (unsigned)f.S);
    float * ws = f.ws;
    int * tickets = reinterpret_cast<int *>(reinterpret_cast<uint8_t *>(f.ws) +
                                            (size_t)f.Hkv * f.T * f.S * G * (128 + 2) * 4);
    switch (G) {
        case 1: return alb_launch(k_flash_attn<1>, grid, dim3(128), 0, st, f.pdl, f.q, f.kc, f.vc, f.Hq, f.Hkv, f.T, f.pos0, f.pos_dev, f.scale, f.S, ws, tickets, f.out);
        case 2: return alb_launch(k_flash_attn<2>, grid, dim3(128), 0, st, f.pdl, f.q, f.kc, f.vc, f.Hq, f.Hkv, f.T, f.pos0, f.pos_dev, f.scale, f.S, ws, tickets, f.out);
        case 4: return alb_launch(k_flash_attn<4>, grid, dim3(128), 0, st, f.pdl, f.q, f.kc, f.vc, f.Hq, f.Hkv, f.T, f.pos0, f.pos_dev, f.scale, f.S, ws, tickets, f.out);
        case 8: return alb_launch(k_flash_attn<8>, grid, dim3(128), 0, st, f.pdl, f.q, f.kc, f.vc, f.Hq, f.Hkv, f.T, f.pos0, f.pos_dev, f.scale, f.S, ws, tickets, f.out);
        default: return cudaErrorInvalidValue;
    }
}

// ------------------------------------------------------------------- argmax
// sample_none / std::max_element (sampler.cpp:34-36): first index of the max.
// Each CTA reduces a contiguous chunk to (value, index); the last CTA (atomic
// ticket) reduces the candidates.  Keys order by value then by LOWER index.
__device__ __forceinline__ unsigned long long am_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);       // order-preserving
    return ((unsigned long long)u << 32) | (uint32_t)(0x7FFFFFFF - idx);
}

__global__ void __launch_bounds__(512)
k_argmax(const float * __restrict__ x, int64_t n, int64_t idx_base, unsigned long long * __restrict__ cand,
         int * __restrict__ ticket, unsigned long long * __restrict__ key_out, int32_t * __restrict__ idx_out) {
    __shared__ unsigned long long red[16];
    __shared__ int last;
    alb_pdl_wait();
    const int64_t chunk = (n + gridDim.x - 1) / gridDim.x;
    const int64_t b0 = (int64_t)blockIdx.x * chunk, b1 = min(n, b0 + chunk);
    unsigned long long best = 0;
    for (int64_t i = b0 + threadIdx.x; i < b1; i += blockDim.x) {
        const unsigned long long k = am_key(x[i], (int)(i + idx_base));
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
        cand[blockIdx.x] = best;
        __threadfence();
        last = (atomicAdd(ticket, 1) == (int)gridDim.x - 1);
    }
    __syncthreads();
    if (!last) { alb_pdl_trigger(); return; }
    __threadfence();
    if (threadIdx.x == 0) {
        unsigned long long b = 0;
        for (unsigned i = 0; i < gridDim.x; ++i) { const unsigned long long k = __ldcg(cand + i); b = k > b ? k : b; }
        if (key_out) *key_out = b;
        if (idx_out) *idx_out = 0x7FFFFFFF - (int32_t)(b & 0xFFFFFFFFu);
        *ticket = 0;
    }
    alb_pdl_trigger();
}

__global__ void k_key_to_index(const unsigned long long * __restrict__ key, int32_t * __restrict__ idx) {
    alb_pdl_wait();
    *idx = 0x7FFFFFFF - (int32_t)(*key & 0xFFFFFFFFu);
    alb_pdl_trigger();
}

cudaError_t launch_argmax(const float * x, int64_t n, int64_t idx_base, void * scratch,
                          unsigned long long * key_out, int32_t * idx_out, bool pdl, cudaStream_t st) {
    const int grid = 64;
    unsigned long long * cand = reinterpret_cast<unsigned long long *>(scratch);
    int * ticket = reinterpret_cast<int *>(cand + grid);
    return alb_launch(k_argmax, dim3(grid), dim3(512), 0, st, pdl, x, n, idx_base, cand, ticket, key_out, idx_out);
}

cudaError_t launch_key_to_index(const unsigned long long * key, int32_t * idx, bool pdl, cudaStream_t st) {
    return alb_launch(k_key_to_index, dim3(1), dim3(1), 0, st, pdl, key, idx);
}

// --------------------------------------------------------- standalone ops
// rms_norm_f32 + MUL (ops.cpp:680-724, binary.cpp): one CTA per row.
__global__ void __launch_bounds__(256)
k_rms_norm(const float * __restrict__ x, const float * __restrict__ w, float * __restrict__ y, int64_t n, float eps) {
    const float * xr = x + (size_t)blockIdx.x * n;
    float * yr = y + (size_t)blockIdx.x * n;
    __shared__ double red[8];
    alb_pdl_wait();
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < n; i += 256) { const float v = xr[i]; s += (double)__fmul_rn(v, v); }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
    const float mean = (float)(t / (double)n);
    const float scale = 1.0f / sqrtf(__fadd_rn(mean, eps));
    for (int64_t i = threadIdx.x; i < n; i += 256) {
        const float v = __fmul_rn(xr[i], scale);
        yr[i] = w ? __fmul_rn(v, w[i]) : v;
    }
    alb_pdl_trigger();
}

// swiglu_f32 (ops.cpp:1038-1092, arm.cpp:1789-1809): y = silu(g) * u
__global__ void k_swiglu(const float * __restrict__ g, const float * __restrict__ u, float * __restrict__ y, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    alb_pdl_wait();
    if (i < n) { const float gv = g[i]; y[i] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), u[i]); }
    alb_pdl_trigger();
}

cudaError_t launch_embed(const uint8_t * Wn, const uint8_t * Ws, int64_t vocab, int64_t E, const int32_t * tokens,
                         int T, float * x, bool pdl, cudaStream_t st) {
    const int64_t n = (int64_t)T * (E / 32);
    return alb_launch(k_embed_q4_0, dim3((unsigned)((n + 127) / 128)), dim3(128), 0, st, pdl, Wn,
                      reinterpret_cast<const uint16_t *>(Ws), q4_scale_pitch(E), tokens, T, E, vocab, x,
                      device_error_ptr());
}

cudaError_t launch_qk_norm_rope_kv(const QkvArgs & a, cudaStream_t st) {
    dim3 grid((unsigned)(a.Hq + 2 * a.Hkv), (unsigned)a.T);
    return alb_launch(k_qk_norm_rope_kv, grid, dim3(128), 0, st, a.pdl, a.qkv, a.qkv_stride, a.Hq, a.Hkv,
                      a.q_norm, a.k_norm, a.eps, a.rope, a.pos0, a.pos_dev, a.q_out, a.kc, a.vc,
                      (int64_t)a.Hkv * 128);
}

cudaError_t launch_rms_norm(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps, bool pdl,
                            cudaStream_t st) {
    return alb_launch(k_rms_norm, dim3((unsigned)rows), dim3(256), 0, st, pdl, x, w, y, n, eps);
}

cudaError_t launch_swiglu(const float * g, const float * u, float * y, int64_t n, bool pdl, cudaStream_t st) {
    return alb_launch(k_swiglu, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, pdl, g, u, y, n);
}

}  // namespace alb
