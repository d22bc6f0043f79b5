// Persistent decode-step kernel: one batch-1 Qwen3 decode token per launch.
//
// Why: a batch-1 decode step streams 2.26 GB of Q4_0 weights (Qwen3-4B) through
// ~250 dependent small operations.  As separate kernels every one pays launch,
// ramp and drain latency (~2 us each) that is larger than its own transfer.
// Here one CTA per SM lives for the whole token:
//   * a producer warp streams this CTA's row shard of every weight matrix of
//     every layer, in consumption order, through an NSLOT x SLOT shared-memory
//     ring with cp.async.bulk (mbarrier completion).  It depends only on free
//     slots, never on activations, so it runs ahead across phase boundaries
//     and keeps HBM busy while the consumers wait at grid barriers;
//   * 8 consumer warps run the graph's phases (reference: build_qwen3_forward_tp,
//     qwen3.cpp:174-275) separated by bounded grid barriers:
//       P1 attn RMSNorm + Q8_0 quantize (per CTA) + fused QKV mat-vec
//       P2 QK-norm + RoPE (+ K/V cache store by the CTA holding the new cell)
//          + attention scores of one (kv head, cell split)
//       P3 global max, softmax numerators, P.V in double, split merge
//       P4 O mat-vec (+ residual)
//       P5 ffn RMSNorm + gate/up mat-vec + SwiGLU
//       P6 down mat-vec (+ residual)
//       P7 final RMSNorm + lm head + argmax (last CTA advances token / position)
// Every operation has the arithmetic of the separate kernels (alb_q4.cu,
// alb_ops.cu), so the result is bit-identical to the multi-kernel engine path.
// All waits (mbarriers, grid barrier) are bounded by %globaltimer; on timeout
// the kernel records ALB_DEVERR_* in the error word and returns.
#include <cfloat>

#include "alb_q4_dev.cuh"
#include "alb_mk.h"

namespace alb {

static constexpr int MK_CONSUMERS = 15;                 // consumer warps (+1 producer = 16 warps, 128 registers)
static constexpr int MK_THREADS = (MK_CONSUMERS + 1) * 32;
static constexpr int MK_NSLOT = 4;
static constexpr uint32_t MK_SLOT = 45 * 1024;
static constexpr int MK_MAX_NB = 384;                   // K <= 12288
static constexpr int MK_UNION_FLOATS = 8192;            // xs records | attention scores
static constexpr int MK_MAX_G = 4;

struct MkShared {
    alignas(128) uint8_t ring[MK_NSLOT][MK_SLOT];
    // GEMV phases use xs (Q8_0 activation records); attention phases use sc
    // (scores / probabilities of this CTA's (kv head, split) item, G x cells)
    union alignas(16) {
        int xs[MK_MAX_NB * XREC_INTS];
        float sc[MK_UNION_FLOATS];
    } u;
    float qs[MK_MAX_G][128];                             // fp16-rounded q of this item
    float ktmp[128];                                     // normed + roped k of the new cell
    double red_d[MK_CONSUMERS];
    double part[MK_CONSUMERS][2];
    float red_f[MK_CONSUMERS][MK_MAX_G];
    uint64_t full[MK_NSLOT], empty[MK_NSLOT];
    int abort_flag;
    int last;
    unsigned long long am;
};
static_assert(MK_MAX_NB * XREC_INTS * 4 <= MK_UNION_FLOATS * 4, "union too small for xs");

__device__ __forceinline__ void mk_bar() {   // the 8 consumer warps only
    asm volatile("bar.sync 1, %0;" :: "n"(MK_CONSUMERS * 32) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned * p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(unsigned * p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned atom_add_release(unsigned * p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.release.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Bounded grid barrier over the consumer warps of all CTAs: arrival is a
// release atomic (the CTA barrier before it makes every consumer thread's
// writes part of the release), the last arrival resets the count and
// publishes the next generation with a release store, the others poll the
// generation with acquire loads.
__device__ bool mk_grid_sync(const MkParams & p, MkShared & sh) {
    mk_bar();
    if (threadIdx.x == 0) {
        const unsigned g = ld_acquire(p.bar_gen);
        if (atom_add_release(p.bar_count, 1u) == (unsigned)gridDim.x - 1) {
            *reinterpret_cast<volatile unsigned *>(p.bar_count) = 0u;
            st_release(p.bar_gen, g + 1);
        } else {
            const uint64_t t0 = alb_globaltimer();
            uint32_t it = 0;
            while (ld_acquire(p.bar_gen) == g) {
                if ((++it & 63) == 0 && alb_globaltimer() - t0 > 2000000000ull) {
                    atomicExch(p.err, ALB_DEVERR_FLAG_TIMEOUT);
                    sh.abort_flag = 1;
                    break;
                }
            }
        }
    }
    mk_bar();
    return sh.abort_flag == 0;
}

// ------------------------------------------------------------ stream plan
// The producer and the consumers walk the same sequence of stages: for each
// matrix stream (per layer: QKV, O, gate/up, down; then the lm head) this
// CTA's contiguous item range, R rows per stage.
struct MkStream {
    const uint8_t * W;
    const uint8_t * S;
    int64_t N, K;
    int unit;      // rows per item (2 for the interleaved gate/up pairs)
};

// Stage plan of a matrix stream: R rows per ring stage.  When a slot holds at
// least one unit per consumer warp, R is a multiple of MK_CONSUMERS units (each
// warp owns whole units, two at a time); otherwise `units` units per stage are
// each split over P warps along K (units * P <= MK_CONSUMERS, as many warps
// busy as possible) and combined through shared memory.
struct MkPlan { int R, units, P; };

__device__ __forceinline__ MkPlan mk_plan(int64_t K, int unit) {
    const int64_t rb = K / 2 + q4_scale_pitch(K) * 2;
    int fit = (int)((int64_t)MK_SLOT / rb) / unit;      // units that fit a slot
    if (fit > 4 * MK_CONSUMERS) fit = 4 * MK_CONSUMERS;
    MkPlan pl;
    if (fit >= MK_CONSUMERS) {
        pl.units = fit / MK_CONSUMERS * MK_CONSUMERS;
        pl.P = 1;
    } else {
        int best_u = 1, best_w = 1;
        for (int u = 1; u <= fit; ++u) {
            const int w = u * (MK_CONSUMERS / u);
            if (w > best_w || (w == best_w && u > best_u)) { best_w = w; best_u = u; }
        }
        pl.units = best_u;
        pl.P = MK_CONSUMERS / best_u;
    }
    pl.R = pl.units * unit;
    return pl;
}

__device__ __forceinline__ int mk_rows_per_stage(int64_t K, int unit) { return mk_plan(K, unit).R; }

__device__ __forceinline__ void mk_range(const MkStream & s, int & r0, int & r1) {
    const int64_t items = s.N / s.unit;
    r0 = (int)(items * blockIdx.x / gridDim.x) * s.unit;
    r1 = (int)(items * (blockIdx.x + 1) / gridDim.x) * s.unit;
}

__device__ __forceinline__ MkStream mk_stream(const MkParams & p, int idx) {
    MkStream s;
    const int l = idx / 4, m = idx % 4;
    if (idx >= 4 * p.n_layer) {
        s.W = p.lm_W; s.S = p.lm_S; s.N = p.V; s.K = p.E; s.unit = 1;
        return s;
    }
    const MkLayer & L = p.layers[l];
    switch (m) {
        case 0: s.W = L.qkv_W; s.S = L.qkv_S; s.N = p.Nqkv; s.K = p.E; s.unit = 1; break;
        case 1: s.W = L.o_W; s.S = L.o_S; s.N = p.E; s.K = p.Dq; s.unit = 1; break;
        case 2: s.W = L.gu_W; s.S = L.gu_S; s.N = 2 * (int64_t)p.F; s.K = p.E; s.unit = 2; break;
        default: s.W = L.dn_W; s.S = L.dn_S; s.N = p.E; s.K = p.F; s.unit = 1; break;
    }
    return s;
}

// Walks the stages of all streams in order (the consumers walk the same list).
struct MkCursor {
    int si = 0, r = 0, r1 = 0, R = 0;
    int64_t rb = 0, sp2 = 0;
    const uint8_t * W = nullptr;
    const uint8_t * S = nullptr;
};

__device__ __forceinline__ bool mk_cursor_next(const MkParams & p, MkCursor & c, int n_streams) {
    c.r += c.R;
    while (c.r >= c.r1) {
        if (c.si >= n_streams) return false;
        const MkStream s = mk_stream(p, c.si++);
        c.R = mk_rows_per_stage(s.K, s.unit);
        mk_range(s, c.r, c.r1);
        c.rb = s.K / 2;
        c.sp2 = q4_scale_pitch(s.K) * 2;
        c.W = s.W;
        c.S = s.S;
    }
    return true;
}

__device__ __forceinline__ void mk_prefetch_stage(const MkCursor & c) {
    const int rows = (c.r1 - c.r) < c.R ? (c.r1 - c.r) : c.R;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;"
                 :: "l"(c.W + (int64_t)c.r * c.rb), "r"((uint32_t)(rows * c.rb)) : "memory");
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;"
                 :: "l"(c.S + (int64_t)c.r * c.sp2), "r"((uint32_t)(rows * c.sp2)) : "memory");
}

// One elected thread: bulk copies of every stage into the ring, and L2
// prefetches of the stages pf_stages ahead, so that HBM keeps streaming
// through the consumers' prologues, barriers and attention.
__device__ void mk_producer(const MkParams & p, MkShared & sh) {
    const int n_streams = 4 * p.n_layer + 1;
    MkCursor cur, ahead;
    for (int k = 0; k < p.pf_stages && mk_cursor_next(p, ahead, n_streams); ++k) mk_prefetch_stage(ahead);
    uint32_t g = 0;
    bool ok = true;
    while (ok && mk_cursor_next(p, cur, n_streams)) {
        const int slot = g % MK_NSLOT;
        if (g >= MK_NSLOT) {
            if (!alb_mbar_wait(&sh.empty[slot], ((g / MK_NSLOT) - 1) & 1) || sh.abort_flag) { ok = false; break; }
        }
        const int rows = (cur.r1 - cur.r) < cur.R ? (cur.r1 - cur.r) : cur.R;
        const uint32_t nb = (uint32_t)(rows * cur.rb), sb = (uint32_t)(rows * cur.sp2);
        alb_mbar_expect_tx(&sh.full[slot], nb + sb);
        alb_bulk_g2s(sh.ring[slot], cur.W + (int64_t)cur.r * cur.rb, nb, &sh.full[slot]);
        alb_bulk_g2s(sh.ring[slot] + (size_t)cur.R * cur.rb, cur.S + (int64_t)cur.r * cur.sp2, sb, &sh.full[slot]);
        if (p.pf_stages > 0 && mk_cursor_next(p, ahead, n_streams)) mk_prefetch_stage(ahead);
        ++g;
    }
    if (!ok) atomicExch(p.err, ALB_DEVERR_MBAR_TIMEOUT);
    // no copy may still be in flight when the CTA exits
    const uint32_t first = g > MK_NSLOT ? g - MK_NSLOT : 0;
    for (uint32_t q = first; q < g; ++q) alb_mbar_wait(&sh.full[q % MK_NSLOT], (q / MK_NSLOT) & 1);
}

// ------------------------------------------------------------ prologues
// RMSNorm (ops.cpp:680-724) * w then Q8_0 (arm.cpp:1819-1853) of an fp32 vector
// into the activation records; w == nullptr: quantize only.  Same arithmetic as
// gemv_prologue_impl (alb_q4.cu).  EMB: the vector is row `token` of the Q4_0
// token table (GET_ROWS, ops.cpp:12-52), dequantized on the fly.
template <bool EMB>
__device__ __forceinline__ float mk_src(const MkParams & p, const float * x, int token, int i) {
    if constexpr (EMB) {
        const int b = i >> 5, j = i & 31;
        const uint8_t byte = p.tok_W[(size_t)token * (p.E / 2) + 16 * b + (j & 15)];
        const float d = alb_h2f(reinterpret_cast<const uint16_t *>(p.tok_S)[(size_t)token * q4_scale_pitch(p.E) + b]);
        return (float)((j < 16 ? (byte & 0x0F) : (byte >> 4)) - 8) * d;
    } else {
        return x[i];
    }
}

// Four consumer threads per 32-value block (a lane quad; thread part k owns
// elements 8k..8k+7): squares summed in double for the RMS, then per block
// the exact max over the quad, d = amax/127 and id = 1/d as IEEE divisions
// (arm.cpp:1834-1851), RNE conversion, and the packed record (8 packed ints,
// fp16-rounded d as float, sum of the q, d as double).
static constexpr int MK_QROUNDS = (MK_MAX_NB * 4 + MK_CONSUMERS * 32 - 1) / (MK_CONSUMERS * 32);

template <bool EMB>
__device__ __forceinline__ void mk_load_quarter(const MkParams & p, const float * x, int token, int q, float * v) {
    if constexpr (EMB) {
        const int b = q >> 2, part = q & 3;
        const uint2 u = *reinterpret_cast<const uint2 *>(p.tok_W + (size_t)token * (p.E / 2) + 16 * b + 8 * (part & 1));
        const float d = alb_h2f(reinterpret_cast<const uint16_t *>(p.tok_S)[(size_t)token * q4_scale_pitch(p.E) + b]);
        const int sh = (part >> 1) * 4;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t w = j < 4 ? u.x : u.y;
            v[j] = (float)((int)((w >> (8 * (j & 3) + sh)) & 0x0F) - 8) * d;
        }
    } else {
        const float4 * s4 = reinterpret_cast<const float4 *>(x + (size_t)q * 8);
        const float4 f0 = s4[0], f1 = s4[1];
        v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
        v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
    }
}

template <bool EMB>
__device__ void mk_quantize(const MkParams & p, const float * x, int token, const float * w, int K, MkShared & sh) {
    constexpr int T = MK_CONSUMERS * 32;
    static_assert(T % 32 == 0, "quads stay inside warps");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nq = K / 8;
    float scale = 1.0f;
    if (w) {   // pass 1: sum of squares (the values are read again in pass 2, from L1)
        double s = 0.0;
        for (int q = tid; q < nq; q += T) {
            float v[8];
            mk_load_quarter<EMB>(p, x, token, q, v);
#pragma unroll
            for (int j = 0; j < 8; ++j) s += (double)__fmul_rn(v[j], v[j]);
        }
        s = alb_warp_sum_d(s);
        if (lane == 0) sh.red_d[warp] = s;
        mk_bar();
        double tot = 0.0;
#pragma unroll
        for (int k = 0; k < MK_CONSUMERS; ++k) tot += sh.red_d[k];
        const float mean = (float)(tot / (double)K);
        scale = 1.0f / sqrtf(__fadd_rn(mean, p.eps));
    }
    for (int k = 0; k < MK_QROUNDS; ++k) {
        const int q = tid + k * T;
        if (q - lane >= nq) break;                       // warp-uniform: no quarter of this warp left
        const bool mine = q < nq;
        float amax = 0.0f;
        float v[8];
        if (mine) {
            mk_load_quarter<EMB>(p, x, token, q, v);
            if (w) {
                const float4 * w4 = reinterpret_cast<const float4 *>(w + (size_t)q * 8);
                const float4 f0 = w4[0], f1 = w4[1];
                const float wv[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], scale), wv[j]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        int sum = 0;
        uint32_t pk[2] = {0u, 0u};
        if (mine) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int qv = __float2int_rn(__fmul_rn(v[j], id));
                sum += qv;
                pk[j >> 2] |= ((uint32_t)qv & 0xFFu) << (8 * (j & 3));
            }
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (mine) {
            int * rec = sh.u.xs + (q >> 2) * XREC_INTS;
            reinterpret_cast<int2 *>(rec)[q & 3] = make_int2((int)pk[0], (int)pk[1]);
            if ((q & 3) == 0) {
                const float dr = alb_h2f(alb_f2h(d));
                const double dd = (double)dr;
                reinterpret_cast<int4 *>(rec)[2] =
                    make_int4(__float_as_int(dr), sum, __double2loint(dd), __double2hiint(dd));
            }
        }
    }
    mk_bar();
}

// ------------------------------------------------------------ mat-vec phase
// Consumes this CTA's stages of stream `s`.  OUT: 0 plain y[row], 1 y[row] +=
// (residual when add_res), 2 SwiGLU pairs y[row/2], 3 logits + argmax key.
template <int OUT>
__device__ __forceinline__ void mk_emit(const MkParams & p, float * y, int row, double a0, double a1, bool add_res,
                                        unsigned long long * best) {
    if constexpr (OUT == 2) {
        y[row / 2] = alb_swiglu1(__double2float_rn(a0), __double2float_rn(a1));
    } else {
        const float yv = __double2float_rn(a0);
        if constexpr (OUT == 3) {
            y[row] = yv;
            uint32_t uu = __float_as_uint(yv);
            uu = (uu & 0x80000000u) ? ~uu : (uu | 0x80000000u);
            const unsigned long long key = ((unsigned long long)uu << 32) | (uint32_t)(0x7FFFFFFF - (row + p.v0));
            *best = key > *best ? key : *best;
        } else if constexpr (OUT == 1) {
            y[row] = add_res ? __fadd_rn(yv, y[row]) : yv;
        } else {
            y[row] = yv;
        }
    }
}

// Dot of one row's blocks [b0, b1) (lane-strided) against the activation
// records; two rows at a time share the record loads.
template <int OUT>
__device__ bool mk_gemv(const MkParams & p, MkShared & sh, const MkStream & s, uint32_t & g, float * y,
                        bool add_res, unsigned long long * best) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const MkPlan pl = mk_plan(s.K, s.unit);
    const int R = pl.R, P = pl.P;
    const int nb = (int)(s.K / 32);
    const int64_t rb = s.K / 2, sp = q4_scale_pitch(s.K);
    int r0, r1;
    mk_range(s, r0, r1);
    int64_t * st_tr = (p.trace && blockIdx.x == 0 && threadIdx.x == 0) ? p.trace + 1024 : nullptr;
    for (int r = r0; r < r1; r += R, ++g) {
        const int slot = g % MK_NSLOT;
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g] = (int64_t)alb_globaltimer();
        if (!alb_mbar_wait(&sh.full[slot], (g / MK_NSLOT) & 1)) {
            if (lane == 0) atomicExch(p.err, ALB_DEVERR_MBAR_TIMEOUT);
            sh.abort_flag = 1;
            return false;
        }
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g + 1] = (int64_t)alb_globaltimer();
        const int n_units = ((r1 - r) < R ? (r1 - r) : R) / s.unit;
        const uint8_t * nib = sh.ring[slot];
        const uint16_t * scl = reinterpret_cast<const uint16_t *>(sh.ring[slot] + (size_t)R * rb);
        if (P == 1) {
            // warp w owns units w, w + W, w + 2W, ...; two per pass
            for (int u0 = warp; u0 < n_units; u0 += 2 * MK_CONSUMERS) {
                const int u1 = u0 + MK_CONSUMERS;
                const bool two = u1 < n_units;
                double a00 = 0.0, a01 = 0.0, a10 = 0.0, a11 = 0.0;
                const int ra = u0 * s.unit, rbw = u1 * s.unit;
                for (int b = lane; b < nb; b += 32) {
                    const int4 * rec = reinterpret_cast<const int4 *>(sh.u.xs + b * XREC_INTS);
                    const int4 a_lo = rec[0], a_hi = rec[1], r2 = rec[2];
                    const double dx = __hiloint2double(r2.w, r2.z);
                    {
                        const uint4 w4 = *reinterpret_cast<const uint4 *>(nib + (size_t)ra * rb + 16 * b);
                        a00 = fma(alb_i2d(q4q8_dot(w4, a_lo, a_hi, r2.y)), dx * alb_h2d(scl[(size_t)ra * sp + b]), a00);
                    }
                    if (s.unit == 2) {
                        const uint4 w4 = *reinterpret_cast<const uint4 *>(nib + (size_t)(ra + 1) * rb + 16 * b);
                        a01 = fma(alb_i2d(q4q8_dot(w4, a_lo, a_hi, r2.y)), dx * alb_h2d(scl[(size_t)(ra + 1) * sp + b]), a01);
                    }
                    if (two) {
                        const uint4 w4 = *reinterpret_cast<const uint4 *>(nib + (size_t)rbw * rb + 16 * b);
                        a10 = fma(alb_i2d(q4q8_dot(w4, a_lo, a_hi, r2.y)), dx * alb_h2d(scl[(size_t)rbw * sp + b]), a10);
                        if (s.unit == 2) {
                            const uint4 w5 = *reinterpret_cast<const uint4 *>(nib + (size_t)(rbw + 1) * rb + 16 * b);
                            a11 = fma(alb_i2d(q4q8_dot(w5, a_lo, a_hi, r2.y)), dx * alb_h2d(scl[(size_t)(rbw + 1) * sp + b]), a11);
                        }
                    }
                }
                a00 = alb_warp_sum_d(a00);
                if (s.unit == 2) a01 = alb_warp_sum_d(a01);
                if (two) {
                    a10 = alb_warp_sum_d(a10);
                    if (s.unit == 2) a11 = alb_warp_sum_d(a11);
                }
                if (lane == 0) {
                    mk_emit<OUT>(p, y, r + ra, a00, a01, add_res, best);
                    if (two) mk_emit<OUT>(p, y, r + rbw, a10, a11, add_res, best);
                }
            }
        } else {
            // unit warp / P, block part warp % P
            const int u = warp / P, part = warp % P;
            if (u < n_units) {
                const int b0 = nb * part / P, b1 = nb * (part + 1) / P;
                const int rl = u * s.unit;
                double acc0 = 0.0, acc1 = 0.0;
                for (int b = b0 + lane; b < b1; b += 32) {
                    const int4 * rec = reinterpret_cast<const int4 *>(sh.u.xs + b * XREC_INTS);
                    const int4 a_lo = rec[0], a_hi = rec[1], r2 = rec[2];
                    const double dx = __hiloint2double(r2.w, r2.z);
                    const uint4 w4 = *reinterpret_cast<const uint4 *>(nib + (size_t)rl * rb + 16 * b);
                    acc0 = fma(alb_i2d(q4q8_dot(w4, a_lo, a_hi, r2.y)), dx * alb_h2d(scl[(size_t)rl * sp + b]), acc0);
                    if (s.unit == 2) {
                        const uint4 w5 = *reinterpret_cast<const uint4 *>(nib + (size_t)(rl + 1) * rb + 16 * b);
                        acc1 = fma(alb_i2d(q4q8_dot(w5, a_lo, a_hi, r2.y)), dx * alb_h2d(scl[(size_t)(rl + 1) * sp + b]), acc1);
                    }
                }
                acc0 = alb_warp_sum_d(acc0);
                if (s.unit == 2) acc1 = alb_warp_sum_d(acc1);
                if (lane == 0) { sh.part[warp][0] = acc0; sh.part[warp][1] = acc1; }
            }
            mk_bar();
            if (warp < n_units && lane == 0) {
                double a0 = 0.0, a1 = 0.0;
                for (int k = 0; k < P; ++k) { a0 += sh.part[warp * P + k][0]; a1 += sh.part[warp * P + k][1]; }
                mk_emit<OUT>(p, y, r + warp * s.unit, a0, a1, add_res, best);
            }
            mk_bar();
        }
        __syncwarp();
        if (lane == 0) alb_mbar_arrive(&sh.empty[slot]);
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g + 2] = (int64_t)alb_globaltimer();
    }
    return true;
}

// ------------------------------------------------------------ attention
// Per-head QK RMSNorm * w + NEOX RoPE of one 128-vector with one warp (lane
// owns dims 4*lane..4*lane+3), same arithmetic as k_qk_norm_rope_kv.
__device__ void mk_norm_rope(const float * src, const float * w, float eps, const float2 * rope_p, float * dst,
                             MkShared & sh, int warp_slot) {
    const int lane = threadIdx.x & 31;
    float v[4];
    double s = 0.0;
#pragma unroll
    for (int e = 0; e < 4; ++e) { v[e] = src[4 * lane + e]; s += (double)__fmul_rn(v[e], v[e]); }
    // 128 fp32 squares: any double summation order is exact in practice (same as the kernel)
    s = alb_warp_sum_d(s);
    const float mean = (float)(s / 128.0);
    const float scale = 1.0f / sqrtf(__fadd_rn(mean, eps));
    float * buf = dst;   // scratch of 128 floats owned by this warp
#pragma unroll
    for (int e = 0; e < 4; ++e) buf[4 * lane + e] = __fmul_rn(__fmul_rn(v[e], scale), w[4 * lane + e]);
    __syncwarp();
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int d = 4 * lane + e;
        const float2 cs = rope_p[d & 63];
        o[e] = d < 64 ? __fsub_rn(__fmul_rn(buf[d], cs.x), __fmul_rn(buf[d + 64], cs.y))
                      : __fadd_rn(__fmul_rn(buf[d - 64], cs.y), __fmul_rn(buf[d], cs.x));
    }
    __syncwarp();
#pragma unroll
    for (int e = 0; e < 4; ++e) buf[4 * lane + e] = o[e];
    __syncwarp();
    (void)sh; (void)warp_slot;
}

__device__ __forceinline__ void mk_split(int n, int S, int s, int & c0, int & c1) {
    const int sz = (n + S - 1) / S;
    c0 = s * sz;
    c1 = min(n, c0 + sz);
    if (c0 > n) c0 = n;
}

// Attention of the new token, one (kv head h, cell split s) item per CTA
// (Hkv * S <= gridDim.x).  Same arithmetic as k_fa_scores / k_fa_pv:
//   QK-norm + RoPE of the G q heads (and of k, stored with v into the cache by
//   the split holding the new cell); scores s_c = fp32 fma chain * scale;
//   split max -> the S CTAs of head h wait for one another (bounded; all CTAs
//   are co-resident under the cooperative launch) -> global max M;
//   p_c = v_expf(s_c - M); L and O = sum_c p_c V_c in double, V staged in
//   shared memory; the last split (ticket) adds the S split records in split
//   order and writes att.
static constexpr int MK_ATT_MAX_CELLS = 512;            // cells per split
static constexpr int MK_VTILE = 64;                     // V rows per shared tile
static_assert(MK_MAX_G * MK_ATT_MAX_CELLS + MK_VTILE * 64 <= MK_UNION_FLOATS, "attention scratch too large");
static_assert(MK_MAX_G * 128 <= 2 * MK_CONSUMERS * 32, "two (g, d) outputs per thread");

// Barrier of the S CTAs of one kv head (same protocol as mk_grid_sync on the
// head's own count / generation words).
__device__ bool mk_group_sync(const MkParams & p, MkShared & sh, unsigned * count, unsigned * gen, unsigned S) {
    mk_bar();
    if (threadIdx.x == 0) {
        const unsigned g = ld_acquire(gen);
        if (atom_add_release(count, 1u) == S - 1) {
            *reinterpret_cast<volatile unsigned *>(count) = 0u;
            st_release(gen, g + 1);
        } else {
            const uint64_t t0 = alb_globaltimer();
            uint32_t it = 0;
            while (ld_acquire(gen) == g) {
                if ((++it & 63) == 0 && alb_globaltimer() - t0 > 2000000000ull) {
                    atomicExch(p.err, ALB_DEVERR_FLAG_TIMEOUT);
                    sh.abort_flag = 1;
                    break;
                }
            }
        }
    }
    mk_bar();
    return sh.abort_flag == 0;
}

template <int G>
__device__ bool mk_attention(const MkParams & p, MkShared & sh, const MkLayer & L, int pos, int layer) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int item = blockIdx.x;
    if (item >= p.Hkv * p.S) return true;
    int64_t * ft = (p.trace && item == 0 && tid == 0 && layer < 36) ? p.trace + 640 + 8 * layer : nullptr;
#define MK_FT(k) do { if (ft) ft[k] = (int64_t)alb_globaltimer(); } while (0)
    MK_FT(0);
    const int n = pos + 1;
    const int64_t row = (int64_t)p.Hkv * 128;
    const int h = item / p.S, s = item % p.S;
    int c0, c1;
    mk_split(n, p.S, s, c0, c1);
    const int nc = c1 - c0;
    const float2 * rp = reinterpret_cast<const float2 *>(p.rope) + (size_t)pos * 64;
    float * sc = sh.u.sc;                                                            // [G][MK_ATT_MAX_CELLS]
    uint16_t * vt = reinterpret_cast<uint16_t *>(sh.u.sc + MK_MAX_G * MK_ATT_MAX_CELLS);  // [MK_VTILE][128]
    for (int g = warp; g < G; g += MK_CONSUMERS) {
        mk_norm_rope(p.qkv + (size_t)(h * G + g) * 128, L.qn, p.eps, rp, sh.qs[g], sh, g);
#pragma unroll
        for (int e = 0; e < 4; ++e) sh.qs[g][4 * lane + e] = __half2float(__float2half_rn(sh.qs[g][4 * lane + e]));
    }
    if (c0 < n && c1 == n && warp == MK_CONSUMERS - 1) {
        mk_norm_rope(p.qkv + (size_t)(p.Hq + h) * 128, L.kn, p.eps, rp, sh.ktmp, sh, 0);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = 4 * lane + e;
            L.kc[(size_t)pos * row + h * 128 + d] = alb_f2h(sh.ktmp[d]);
            L.vc[(size_t)pos * row + h * 128 + d] = alb_f2h(p.qkv[(size_t)(p.Hq + p.Hkv + h) * 128 + d]);
        }
    }
    mk_bar();   // q in smem; the new K/V cell is stored (visible to this CTA)
    // scores: one thread per cell, K row read as 16 x 16 B
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; ++g) mx[g] = -INFINITY;
    for (int c = c0 + tid; c < c1; c += MK_CONSUMERS * 32) {
        const uint4 * kr = reinterpret_cast<const uint4 *>(L.kc + (size_t)c * row + (size_t)h * 128);
        float a[G];
#pragma unroll
        for (int g = 0; g < G; ++g) a[g] = 0.0f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            uint4 kv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) kv[j] = __ldcg(kr + 8 * half + j);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t wd[4] = {kv[j].x, kv[j].y, kv[j].z, kv[j].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 kf = __half22float2(*reinterpret_cast<const __half2 *>(&wd[e]));
                    const int d = 64 * half + 8 * j + 2 * e;
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        a[g] = __fmaf_rn(kf.x, sh.qs[g][d], a[g]);
                        a[g] = __fmaf_rn(kf.y, sh.qs[g][d + 1], a[g]);
                    }
                }
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float v = __fmul_rn(a[g], p.scale);
            sc[g * MK_ATT_MAX_CELLS + (c - c0)] = v;
            mx[g] = fmaxf(mx[g], v);
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float m = alb_warp_max(mx[g]);
        if (lane == 0) sh.red_f[warp][g] = m;
    }
    mk_bar();
    if (tid < G) {
        float m = -INFINITY;
        for (int k = 0; k < MK_CONSUMERS; ++k) m = fmaxf(m, sh.red_f[k][tid]);
        __stcg(p.smax + ((size_t)h * p.S + s) * G + tid, m);
    }
    MK_FT(1);
    if (!mk_group_sync(p, sh, p.grp + 2 * h, p.grp + 2 * h + 1, (unsigned)p.S)) return false;
    MK_FT(2);
    if (tid < G) {
        float m = -INFINITY;
        for (int k = 0; k < p.S; ++k) m = fmaxf(m, __ldcg(p.smax + ((size_t)h * p.S + k) * G + tid));
        sh.red_f[0][tid] = m;
    }
    mk_bar();
    for (int i = tid; i < G * nc; i += MK_CONSUMERS * 32) {
        const int g = i / nc, c = i - g * nc;
        float & sref = sc[g * MK_ATT_MAX_CELLS + c];
        sref = alb_ref_expf(__fsub_rn(sref, sh.red_f[0][g]));
    }
    MK_FT(3);
    // P.V: thread (g, d) owns output d of q head g; cells summed in order in double
    double O[2] = {0.0, 0.0};
    for (int t0 = 0; t0 < nc; t0 += MK_VTILE) {
        const int tn = min(MK_VTILE, nc - t0);
        mk_bar();   // numerators written / previous tile consumed
        for (int i = tid; i < tn * 16; i += MK_CONSUMERS * 32) {
            const int c = i >> 4, j = i & 15;
            reinterpret_cast<uint4 *>(vt)[i] =
                __ldcg(reinterpret_cast<const uint4 *>(L.vc + (size_t)(c0 + t0 + c) * row + (size_t)h * 128) + j);
        }
        mk_bar();
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int i = tid + q * MK_CONSUMERS * 32;
            if (i < G * 128) {
                const int g = i >> 7, d = i & 127;
                const float * pg = sc + g * MK_ATT_MAX_CELLS + t0;
                double o = O[q];
                for (int c = 0; c < tn; ++c) o = fma((double)pg[c], (double)alb_h2f(vt[c * 128 + d]), o);
                O[q] = o;
            }
        }
    }
    MK_FT(4);
    // split record [h][s][G][129] doubles: O[0..127], L
    double * rec = p.part + ((size_t)h * p.S + s) * G * 129;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const int i = tid + q * MK_CONSUMERS * 32;
        if (i < G * 128) {
            const int g = i >> 7, d = i & 127;
            __stcg(rec + g * 129 + d, O[q]);
            if (d == 0) {
                double l = 0.0;
                for (int c = 0; c < nc; ++c) l += (double)sc[g * MK_ATT_MAX_CELLS + c];
                __stcg(rec + g * 129 + 128, l);
            }
        }
    }
    __threadfence();
    mk_bar();
    if (tid == 0) sh.last = (atomicAdd(&p.tickets[h], 1) == p.S - 1);
    mk_bar();
    if (sh.last) {
        __threadfence();
        const double * hb = p.part + (size_t)h * p.S * G * 129;
        for (int i = tid; i < G * 128; i += MK_CONSUMERS * 32) {
            const int g = i >> 7, d = i & 127;
            double Lt = 0.0, Ot = 0.0;
            for (int k = 0; k < p.S; ++k) {
                const double * pk = hb + ((size_t)k * G + g) * 129;
                Lt += __ldcg(pk + 128);
                Ot += __ldcg(pk + d);
            }
            p.att[(size_t)(h * G + g) * 128 + d] = Lt > 0.0 ? __double2float_rn(Ot / Lt) : 0.0f;
        }
        if (tid == 0) p.tickets[h] = 0;
    }
    MK_FT(5);
#undef MK_FT
    return true;
}

// ------------------------------------------------------------ the kernel
template <int G>
__global__ void __launch_bounds__(MK_THREADS, 1)
k_decode_step(const MkParams p) {
    extern __shared__ __align__(128) uint8_t mk_smem[];
    MkShared & sh = *reinterpret_cast<MkShared *>(mk_smem);
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        for (int i = 0; i < MK_NSLOT; ++i) { alb_mbar_init(&sh.full[i], 1); alb_mbar_init(&sh.empty[i], MK_CONSUMERS); }
        sh.abort_flag = 0;
        sh.am = 0ull;
        alb_mbar_fence_init();
    }
    __syncthreads();
    if (warp == MK_CONSUMERS) {
        if ((tid & 31) == 0) mk_producer(p, sh);
        return;
    }
    const int pos = p.pos[0];
    const int token = p.tok[0];
    uint32_t g = 0;
    bool ok = true;
    {   // embedding: the CTA stores the x rows it owns (its O / down output range)
        const MkStream so = mk_stream(p, 1);
        int r0, r1;
        mk_range(so, r0, r1);
        for (int i = r0 + tid; i < r1; i += MK_CONSUMERS * 32) p.x[i] = mk_src<true>(p, nullptr, token, i);
    }
    int64_t * tr = (p.trace && blockIdx.x == 0 && tid == 0) ? p.trace : nullptr;
    int tn = 0;
#define MK_TRACE() do { if (tr && tn < 1024) tr[tn++] = (int64_t)alb_globaltimer(); } while (0)
    MK_TRACE();
    for (int l = 0; l < p.n_layer && ok; ++l) {
        const MkLayer & L = p.layers[l];
        // P1: attn norm + QKV
        if (l == 0) mk_quantize<true>(p, nullptr, token, L.an, p.E, sh);
        else mk_quantize<false>(p, p.x, 0, L.an, p.E, sh);
        MK_TRACE();
        ok = mk_gemv<0>(p, sh, mk_stream(p, 4 * l + 0), g, p.qkv, false, nullptr);
        MK_TRACE();
        if (!ok || !mk_grid_sync(p, sh)) { ok = false; break; }
        MK_TRACE();
        // P2+P3: attention of the new token
        if (!mk_attention<G>(p, sh, L, pos, l)) { ok = false; break; }
        MK_TRACE();
        MK_TRACE();
        MK_TRACE();
        if (!mk_grid_sync(p, sh)) { ok = false; break; }
        MK_TRACE();
        // P4: O projection + residual
        mk_quantize<false>(p, p.att, 0, nullptr, p.Dq, sh);
        MK_TRACE();
        ok = mk_gemv<1>(p, sh, mk_stream(p, 4 * l + 1), g, p.x, p.rank == 0, nullptr);
        MK_TRACE();
        if (!ok || !mk_grid_sync(p, sh)) { ok = false; break; }
        MK_TRACE();
        // P5: ffn norm + gate/up + SwiGLU
        mk_quantize<false>(p, p.x, 0, L.fn, p.E, sh);
        MK_TRACE();
        ok = mk_gemv<2>(p, sh, mk_stream(p, 4 * l + 2), g, p.h, false, nullptr);
        MK_TRACE();
        if (!ok || !mk_grid_sync(p, sh)) { ok = false; break; }
        MK_TRACE();
        // P6: down projection + residual
        mk_quantize<false>(p, p.h, 0, nullptr, p.F, sh);
        MK_TRACE();
        ok = mk_gemv<1>(p, sh, mk_stream(p, 4 * l + 3), g, p.x, p.rank == 0, nullptr);
        MK_TRACE();
        if (!ok || !mk_grid_sync(p, sh)) { ok = false; break; }
        MK_TRACE();
    }
    if (!ok) return;
    // P7: output norm + lm head + argmax
    mk_quantize<false>(p, p.x, 0, p.out_norm, p.E, sh);
    MK_TRACE();
    unsigned long long best = 0ull;
    if (!mk_gemv<3>(p, sh, mk_stream(p, 4 * p.n_layer), g, p.logits, false, &best)) return;
    MK_TRACE();
#undef MK_TRACE
    // CTA argmax over the warps' candidates
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if ((tid & 31) == 0) atomicMax(&sh.am, best);
    mk_bar();
    if (tid == 0) {
        p.cand[blockIdx.x] = sh.am;
        __threadfence();
        sh.last = (atomicAdd(p.am_ticket, 1) == (int)gridDim.x - 1);
    }
    mk_bar();
    if (sh.last && tid == 0) {
        __threadfence();
        unsigned long long b = 0ull;
        for (unsigned i = 0; i < gridDim.x; ++i) { const unsigned long long k = __ldcg(p.cand + i); b = k > b ? k : b; }
        const int32_t nxt = 0x7FFFFFFF - (int32_t)(b & 0xFFFFFFFFu);
        *p.next = nxt;
        if (p.advance) {
            const int32_t st = *p.step;
            if (st < p.gen_cap) p.gen_out[st] = nxt;
            *p.step = st + 1;
            *p.tok = nxt;
            *p.pos = pos + 1;
        }
        *p.am_ticket = 0;
    }
}

size_t mk_smem_bytes() { return sizeof(MkShared); }

cudaError_t launch_decode_step(const MkParams & p, cudaStream_t st) {
    const size_t smem = sizeof(MkShared);
    static size_t attr[9] = {0};
    auto go = [&](auto kern, int gi) -> cudaError_t {
        if (attr[gi] != smem) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
            attr[gi] = smem;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)p.ncta);
        cfg.blockDim = dim3(MK_THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = st;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeCooperative;
        at[0].val.cooperative = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kern, p);
    };
    switch (p.Hq / p.Hkv) {
        case 1: return go(k_decode_step<1>, 1);
        case 2: return go(k_decode_step<2>, 2);
        case 4: return go(k_decode_step<4>, 4);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace alb
