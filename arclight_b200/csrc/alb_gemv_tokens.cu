// Token-batched Q4_0 x Q8_0 mat-vec for prefill ubatches (T > 1): each warp
// streams one weight row (or a gate/up row pair) once and dots it with up to
// TB = 8 tokens' Q8_0 activations held in shared memory.  Same per-block
// arithmetic as the batch-1 kernel (reference: forward_mul_mat with ne11 > 3,
// arm.cpp:1911-1917, gemm.cpp:495-974, which computes per row and token the
// same int32 block dots and fp32 scale products).
#include "alb_q4_dev.cuh"

namespace alb {

static constexpr int TB = 8;

template <int IN>
__device__ __forceinline__ void tokens_prologue(const GemvArgs & a, int * xs, int nb, int tb) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ double red[GEMV_WARPS];
    for (int t = 0; t < tb; ++t) {
        const float * x = static_cast<const float *>(a.x) + (size_t)t * a.x_stride;
        float scale = 1.0f;
        if constexpr (IN == GEMV_IN_F32_RMS) {
            double s = 0.0;
            for (int i = tid; i < a.K; i += GEMV_WARPS * 32) { const float v = x[i]; s += (double)__fmul_rn(v, v); }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            __syncthreads();
            if (lane == 0) red[warp] = s;
            __syncthreads();
            double tot = 0.0;
#pragma unroll
            for (int w = 0; w < GEMV_WARPS; ++w) tot += red[w];
            const float mean = (float)(tot / (double)a.K);
            scale = 1.0f / sqrtf(__fadd_rn(mean, a.eps));
        }
        int * xt = xs + (size_t)t * nb * XREC_INTS;
        for (int b = warp; b < nb; b += GEMV_WARPS) {
            float v = x[b * 32 + lane];
            if constexpr (IN == GEMV_IN_F32_RMS) v = __fmul_rn(__fmul_rn(v, scale), a.norm_w[b * 32 + lane]);
            int8_t q; uint16_t dh;
            q8_block_lane(v, q, dh);
            store_xrec(xt, b, lane, q, dh);
        }
    }
}

template <int ITERS, int RPW, int IN, int OUT>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
k_gemv_tokens(const GemvArgs a, int tb) {
    extern __shared__ int4 smem_i4[];
    int * xs = reinterpret_cast<int *>(smem_i4);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = (int)(a.K / 32);
    const size_t row_bytes = (size_t)a.K / 2;
    const int64_t sp = q4_scale_pitch(a.K);
    const uint16_t * Ws = reinterpret_cast<const uint16_t *>(a.S);
    const int64_t n_items = a.N / RPW;
    alb_pdl_wait();
    tokens_prologue<IN>(a, xs, nb, tb);
    __syncthreads();
    alb_pdl_trigger();
    for (int64_t item = (int64_t)blockIdx.x * GEMV_WARPS + warp; item < n_items; item += (int64_t)gridDim.x * GEMV_WARPS) {
        double acc[TB][RPW];
#pragma unroll
        for (int t = 0; t < TB; ++t)
#pragma unroll
            for (int r = 0; r < RPW; ++r) acc[t][r] = 0.0;
#pragma unroll
        for (int i = 0; i < ITERS; ++i) {
            const int b = lane + 32 * i;
            if (b < nb) {
                uint4 w[RPW];
                float dw[RPW];
#pragma unroll
                for (int r = 0; r < RPW; ++r) {
                    const int64_t row = item * RPW + r;
                    w[r] = alb_ld_stream(a.W + row * row_bytes + 16 * b);
                    dw[r] = alb_h2f(__ldg(Ws + row * sp + b));
                }
#pragma unroll
                for (int t = 0; t < TB; ++t) {
                    if (t < tb) {
                        const int4 * rec = reinterpret_cast<const int4 *>(xs + ((size_t)t * nb + b) * XREC_INTS);
                        const int4 a_lo = rec[0], a_hi = rec[1];
                        const int2 ds = reinterpret_cast<const int2 *>(rec + 2)[0];
                        const float dx = __int_as_float(ds.x);
#pragma unroll
                        for (int r = 0; r < RPW; ++r) {
                            const int I = q4q8_dot(w[r], a_lo, a_hi, ds.y);
                            acc[t][r] = fma((double)I, (double)__fmul_rn(dx, dw[r]), acc[t][r]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            if (t >= tb) break;
#pragma unroll
            for (int r = 0; r < RPW; ++r) acc[t][r] = alb_warp_sum_d(acc[t][r]);
            if (lane == 0) {
                float * yt = a.y + (size_t)t * a.y_stride;
                if constexpr (OUT == GEMV_OUT_SWIGLU) {
                    const float g = __double2float_rn(acc[t][0]), u = __double2float_rn(acc[t][1]);
                    yt[item] = alb_swiglu1(g, u);
                } else {
                    const float * rt = a.residual ? a.residual + (size_t)t * a.y_stride : nullptr;
#pragma unroll
                    for (int r = 0; r < RPW; ++r) {
                        const int64_t row = item * RPW + r;
                        const float yv = __double2float_rn(acc[t][r]);
                        yt[row] = rt ? __fadd_rn(yv, rt[row]) : yv;
                    }
                }
            }
        }
    }
}

template <int ITERS, int RPW, int IN, int OUT>
static cudaError_t launch_tokens_t(const GemvArgs & a, int tb, cudaStream_t st) {
    auto kern = k_gemv_tokens<ITERS, RPW, IN, OUT>;
    const size_t smem = (size_t)TB * (a.K / 32) * XREC_INTS * 4;
    static size_t attr = 0;
    if (smem > 48 * 1024 && smem > attr) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr = smem;
    }
    int occ = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, GEMV_WARPS * 32, smem);
    if (occ < 1) occ = 1;
    const int64_t items = a.N / RPW;
    int64_t grid = (int64_t)alb_sm_count() * occ;
    if (grid * GEMV_WARPS > items) grid = (items + GEMV_WARPS - 1) / GEMV_WARPS;
    return alb_launch(kern, dim3((unsigned)grid), dim3(GEMV_WARPS * 32), smem, st, a.pdl, a, tb);
}

template <int IN, int OUT>
static cudaError_t dispatch_tokens(const GemvArgs & a, int tb, cudaStream_t st) {
    constexpr int RPW = OUT == GEMV_OUT_SWIGLU ? 2 : 1;
    switch ((int)((a.K / 32 + 31) / 32)) {
        case 1: return launch_tokens_t<1, RPW, IN, OUT>(a, tb, st);
        case 2: return launch_tokens_t<2, RPW, IN, OUT>(a, tb, st);
        case 3: return launch_tokens_t<3, RPW, IN, OUT>(a, tb, st);
        case 4: return launch_tokens_t<4, RPW, IN, OUT>(a, tb, st);
        case 5: case 6: return launch_tokens_t<6, RPW, IN, OUT>(a, tb, st);
        case 7: case 8: return launch_tokens_t<8, RPW, IN, OUT>(a, tb, st);
        case 9: case 10: return launch_tokens_t<10, RPW, IN, OUT>(a, tb, st);
        case 11: case 12: return launch_tokens_t<12, RPW, IN, OUT>(a, tb, st);
        default: return cudaErrorInvalidValue;
    }
}

// T tokens: rows of x at x_stride floats, rows of y at y_stride floats.
cudaError_t launch_gemv_tokens(const GemvArgs & a_in, int64_t T, cudaStream_t st) {
    if (a_in.in_mode == GEMV_IN_Q8 || a_in.out_mode == GEMV_OUT_DOTS) return cudaErrorInvalidValue;
    for (int64_t t0 = 0; t0 < T; t0 += TB) {
        GemvArgs a = a_in;
        const int tb = (int)((T - t0) < TB ? (T - t0) : TB);
        a.x = static_cast<const float *>(a_in.x) + (size_t)t0 * a_in.x_stride;
        a.y = a_in.y + (size_t)t0 * a_in.y_stride;
        a.residual = a_in.residual ? a_in.residual + (size_t)t0 * a_in.y_stride : nullptr;
        cudaError_t e;
        if (a.in_mode == GEMV_IN_F32_RMS)
            e = a.out_mode == GEMV_OUT_SWIGLU ? dispatch_tokens<GEMV_IN_F32_RMS, GEMV_OUT_SWIGLU>(a, tb, st)
                                              : dispatch_tokens<GEMV_IN_F32_RMS, GEMV_OUT_PLAIN>(a, tb, st);
        else
            e = a.out_mode == GEMV_OUT_SWIGLU ? dispatch_tokens<GEMV_IN_F32, GEMV_OUT_SWIGLU>(a, tb, st)
                                              : dispatch_tokens<GEMV_IN_F32, GEMV_OUT_PLAIN>(a, tb, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace alb
