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
#include <cstddef>

#include "alb_q4_dev.cuh"
#include "alb_mk.h"

namespace alb {

static constexpr int MK_CONSUMERS = 15;                 // consumer warps (+1 producer = 16 warps, 128 registers)
static constexpr int MK_THREADS = (MK_CONSUMERS + 1) * 32;
static constexpr int MK_NSLOT = 4;
static constexpr uint32_t MK_SLOT = 44 * 1024;          // 30 rows of K = 2560
static constexpr int MK_MAX_NB = 384;                   // K <= 12288
static constexpr int MK_MAX_G = 4;
static constexpr int MK_SC_PITCH = MK_ATT_MAX_CELLS + 4;
static constexpr int MK_KV_TILE = 64;                   // cells staged in shared memory per split
static constexpr int MK_KROW = 136;                     // K tile row pitch (halves): rows on distinct banks
static constexpr int MK_QROW = 132;                     // q row pitch (floats)

// Attention scratch of one (kv head, split) item: K/V cells [c0, c0 + 64), the
// layer's QK-norm weights and the RoPE row are bulk-copied in during the QKV
// phase; scores / probabilities per q head.
struct MkAttSmem {
    // scores (fp32, pitch MK_SC_PITCH, in the first half), then the numerators
    // times 2^1008 (double; see the P.V loop) in place
    double pd[MK_MAX_G][MK_ATT_MAX_CELLS];
    alignas(16) uint16_t kt[MK_KV_TILE][MK_KROW];
    alignas(16) uint16_t vt[MK_KV_TILE][128];
    alignas(16) float qn[128];
    alignas(16) float kn[128];
    alignas(16) float2 rope[64];
};

struct MkShared {
    alignas(128) uint8_t ring[MK_NSLOT][MK_SLOT];
    // GEMV phases use xs (Q8_0 activation records, read into registers at the
    // start of each mat-vec); the attention phase uses a
    union alignas(16) {
        int xs[MK_MAX_NB * XREC_INTS];
        MkAttSmem a;
    } u;
    alignas(16) float qs[MK_MAX_G][MK_QROW];             // fp16-rounded q of this item
    float ktmp[128];                                     // normed + roped k of the new cell
    double red_d[MK_CONSUMERS];
    double part[MK_CONSUMERS][2];
    float red_f[MK_CONSUMERS][MK_MAX_G];
    uint64_t full[MK_NSLOT], empty[MK_NSLOT];
    uint64_t kvbar;                                      // attention staging copies landed
    uint64_t stage_ok;                                   // consumers: the staging region is free
    int abort_flag;
    int last;
    unsigned long long am;
};

// The CTA's shared state, addressed from the extern __shared__ symbol inside
// every function (so the compiler emits shared-space loads and stores, also in
// the non-inlined phase functions, instead of generic ones).
extern __shared__ __align__(128) uint8_t mk_smem[];
__device__ __forceinline__ MkShared & mk_sh() { return *reinterpret_cast<MkShared *>(mk_smem); }

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
__device__ bool mk_grid_sync(const MkParams & p, MkShared & sh_arg) {
    MkShared & sh = mk_sh();
    (void)sh_arg;
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

static constexpr int MK_RECS = 4;                       // activation records per lane (128 blocks per warp)

__device__ __forceinline__ MkPlan mk_plan(int64_t K, int unit) {
    const int64_t rb = K / 2 + q4_scale_pitch(K) * 2;
    const int nb = (int)(K / 32);
    const int pmin = (nb + 32 * MK_RECS - 1) / (32 * MK_RECS);
    int fit = (int)((int64_t)MK_SLOT / rb) / unit;      // units that fit a slot
    if (fit > 4 * MK_CONSUMERS) fit = 4 * MK_CONSUMERS;
    MkPlan pl;
    if (fit >= MK_CONSUMERS && pmin == 1) {
        pl.units = fit / MK_CONSUMERS * MK_CONSUMERS;
        pl.P = 1;
    } else {
        int best_u = 1, best_w = 0;
        for (int u = 1; u <= fit && u * pmin <= MK_CONSUMERS; ++u) {
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
__device__ void mk_producer(const MkParams & p, MkShared & sh_arg) {
    MkShared & sh = mk_sh();
    (void)sh_arg;
    const int n_streams = 4 * p.n_layer + 1;
    MkCursor cur, ahead;
    for (int k = 0; k < p.pf_stages && mk_cursor_next(p, ahead, n_streams); ++k) mk_prefetch_stage(ahead);
    uint32_t g = 0;
    bool ok = true;
    while (ok && mk_cursor_next(p, cur, n_streams)) {
        const int slot = g % MK_NSLOT;
        if (g >= MK_NSLOT) {
            if (!alb_mbar_wait_backoff(&sh.empty[slot], ((g / MK_NSLOT) - 1) & 1) || sh.abort_flag) { ok = false; break; }
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
// gemv_prologue_impl (alb_q4.cu).  The embedding (GET_ROWS, ops.cpp:12-52) is
// row `token` of the Q4_0 token table, dequantized on the fly.
__device__ __forceinline__ float mk_embed(const MkParams & p, int token, int i) {
    const int b = i >> 5, j = i & 31;
    const uint8_t byte = p.tok_W[(size_t)token * (p.E / 2) + 16 * b + (j & 15)];
    const float d = alb_h2f(reinterpret_cast<const uint16_t *>(p.tok_S)[(size_t)token * q4_scale_pitch(p.E) + b]);
    return (float)((j < 16 ? (byte & 0x0F) : (byte >> 4)) - 8) * d;
}

// Four consumer threads per 32-value block (a lane quad; thread part k owns
// elements 8k..8k+7): squares summed in double for the RMS, then per block
// the exact max over the quad, d = amax/127 and id = 1/d as IEEE divisions
// (arm.cpp:1834-1851), RNE conversion, and the packed record (8 packed ints,
// fp16-rounded d as float, sum of the q, d as double).
static constexpr int MK_QROUNDS = (MK_MAX_NB * 4 + MK_CONSUMERS * 32 - 1) / (MK_CONSUMERS * 32);

__device__ __forceinline__ void mk_load_quarter(const MkParams & p, const float * x, int token, int q, float * v) {
    if (x == nullptr) {   // row `token` of the Q4_0 token table
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

// x == nullptr: the vector is row `token` of the token table (the embedding).
__device__ __noinline__ void mk_quantize(const MkParams & p, const float * x, int token, const float * w, int K, MkShared & sh_arg) {
    MkShared & sh = mk_sh();
    (void)sh_arg;
    constexpr int T = MK_CONSUMERS * 32;
    static_assert(T % 32 == 0, "quads stay inside warps");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nq = K / 8;
    float scale = 1.0f;
    if (w) {   // pass 1: sum of squares (the values are read again in pass 2, from L1)
        double s = 0.0;
        for (int q = tid; q < nq; q += T) {
            float v[8];
            mk_load_quarter(p, x, token, q, v);
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
            mk_load_quarter(p, x, token, q, v);
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
__device__ __forceinline__ void mk_emit(int OUT, const MkParams & p, float * y, int row, double a0, double a1, bool add_res,
                                        unsigned long long * best) {
    if (OUT == 2) {
        y[row / 2] = alb_swiglu1(__double2float_rn(a0), __double2float_rn(a1));
    } else {
        const float yv = __double2float_rn(a0);
        if (OUT == 3) {
            y[row] = yv;
            uint32_t uu = __float_as_uint(yv);
            uu = (uu & 0x80000000u) ? ~uu : (uu | 0x80000000u);
            const unsigned long long key = ((unsigned long long)uu << 32) | (uint32_t)(0x7FFFFFFF - (row + p.v0));
            *best = key > *best ? key : *best;
        } else if (OUT == 1) {
            y[row] = add_res ? __fadd_rn(yv, y[row]) : yv;
        } else {
            y[row] = yv;
        }
    }
}

// Each lane holds the activation records of its blocks in registers for the
// whole stream (P == 1: blocks lane + 32k; P > 1: the warp's K part
// [b0, b1), lane-strided).  A pass reduces two rows at once.
__device__ __forceinline__ void mk_dot(double & a, const uint8_t * nrow, const uint16_t * srow, int b, int4 lo, int4 hi,
                                       int asum, double dx) {
    const uint4 w4 = *reinterpret_cast<const uint4 *>(nrow + 16 * b);
    a = fma(alb_i2d(q4q8_dot(w4, lo, hi, asum)), dx * alb_h2d(srow[b]), a);
}

// Half-warp form for K <= 2560 (nb <= 80, no K split): each half-warp takes
// one row of a pair (gate/up unit, or rows u and u + 15), 16 lanes x 5 blocks
// of records in registers, a 4-level shuffle reduction per half.
static constexpr int MK_RECS_H = 5;

// KB = blocks per lane = nb / 16 exactly (no per-block predicates); the record
// scale is held pre-multiplied by 2^1008 so the weight scale enters as bits.
template <int KB>
__device__ __noinline__ int64_t mk_gemv_hk(int OUT, const MkParams & p, const MkStream s, uint32_t g, float * y,
                                           bool add_res) {
    MkShared & sh = mk_sh();
    unsigned long long best_key = 0ull;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = lane >> 4, hl = lane & 15;
    const int R = mk_plan(s.K, s.unit).R;
    constexpr int nb = 16 * KB;
    const int64_t rb = s.K / 2, sp = q4_scale_pitch(s.K);
    int4 rlo[KB], rhi[KB];
    int rsum[KB];
    double rdx[KB];
#pragma unroll
    for (int k = 0; k < KB; ++k) {
        const int4 * rec = reinterpret_cast<const int4 *>(sh.u.xs + (hl + 16 * k) * XREC_INTS);
        rlo[k] = rec[0];
        rhi[k] = rec[1];
        const int4 r2 = rec[2];
        rsum[k] = r2.y;
        rdx[k] = __hiloint2double(r2.w, r2.z) * 0x1p1008;   // finite: d <= 65504 < 2^16
    }
    int r0, r1;
    mk_range(s, r0, r1);
    int64_t * st_tr = (p.trace && blockIdx.x == 0 && threadIdx.x == 0) ? p.trace + 1024 : nullptr;
    for (int r = r0; r < r1; r += R, ++g) {
        const int slot = g % MK_NSLOT;
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g] = (int64_t)alb_globaltimer();
        if (!alb_mbar_wait(&sh.full[slot], (g / MK_NSLOT) & 1)) {
            if (lane == 0) atomicExch(p.err, ALB_DEVERR_MBAR_TIMEOUT);
            sh.abort_flag = 1;
            return -1;
        }
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g + 1] = (int64_t)alb_globaltimer();
        const int rows = (r1 - r) < R ? (r1 - r) : R;
        const uint8_t * nib = sh.ring[slot];
        const uint16_t * scl = reinterpret_cast<const uint16_t *>(sh.ring[slot] + (size_t)R * rb);
        for (int i = 0;; ++i) {
            int ra, rc;
            if (s.unit == 2) { ra = 2 * (warp + MK_CONSUMERS * i); rc = ra + 1; }
            else { ra = warp + 2 * MK_CONSUMERS * i; rc = ra + MK_CONSUMERS; }
            if (ra >= rows) break;
            const int row = half ? rc : ra;
            const bool live = row < rows;
            const int rr = live ? row : ra;
            const uint4 * nr = reinterpret_cast<const uint4 *>(nib + (size_t)rr * rb) + hl;
            const uint16_t * sr = scl + (size_t)rr * sp + hl;
            uint4 w[KB];
            uint32_t hs[KB];
#pragma unroll
            for (int k = 0; k < KB; ++k) { w[k] = nr[16 * k]; hs[k] = sr[16 * k]; }
            double a = 0.0;
#pragma unroll
            for (int k = 0; k < KB; ++k)
                a = fma(alb_i2d(q4q8_dot_fast(w[k], rlo[k], rhi[k], rsum[k])), rdx[k] * alb_h2d_bits(hs[k]), a);
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (s.unit == 2) {
                const double up = __shfl_sync(0xffffffffu, a, 16);
                if (lane == 0) mk_emit(OUT, p, y, r + ra, a, up, add_res, &best_key);
            } else if (hl == 0 && live) {
                mk_emit(OUT, p, y, r + row, a, 0.0, add_res, &best_key);
            }
        }
        __syncwarp();
        if (lane == 0) alb_mbar_arrive(&sh.empty[slot]);
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g + 2] = (int64_t)alb_globaltimer();
    }
    if (OUT == 3) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long kk = __shfl_xor_sync(0xffffffffu, best_key, o);
            best_key = kk > best_key ? kk : best_key;
        }
        if (lane == 0) atomicMax(&sh.am, best_key);
    }
    return (int64_t)g;
}

__device__ __noinline__ int64_t mk_gemv_h(int OUT, const MkParams & p, const MkStream s, uint32_t g, float * y,
                                          bool add_res) {
    MkShared & sh = mk_sh();
    unsigned long long best_key = 0ull;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = lane >> 4, hl = lane & 15;
    const int R = mk_plan(s.K, s.unit).R;
    const int nb = (int)(s.K / 32);
    const int64_t rb = s.K / 2, sp = q4_scale_pitch(s.K);
    int4 rlo[MK_RECS_H], rhi[MK_RECS_H];
    int rsum[MK_RECS_H];
    double rdx[MK_RECS_H];
#pragma unroll
    for (int k = 0; k < MK_RECS_H; ++k) {
        const int b = hl + 16 * k;
        const int4 * rec = reinterpret_cast<const int4 *>(sh.u.xs + (b < nb ? b : 0) * XREC_INTS);
        rlo[k] = rec[0];
        rhi[k] = rec[1];
        const int4 r2 = rec[2];
        rsum[k] = r2.y;
        rdx[k] = __hiloint2double(r2.w, r2.z);
    }
    int r0, r1;
    mk_range(s, r0, r1);
    int64_t * st_tr = (p.trace && blockIdx.x == 0 && threadIdx.x == 0) ? p.trace + 1024 : nullptr;
    for (int r = r0; r < r1; r += R, ++g) {
        const int slot = g % MK_NSLOT;
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g] = (int64_t)alb_globaltimer();
        if (!alb_mbar_wait(&sh.full[slot], (g / MK_NSLOT) & 1)) {
            if (lane == 0) atomicExch(p.err, ALB_DEVERR_MBAR_TIMEOUT);
            sh.abort_flag = 1;
            return -1;
        }
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g + 1] = (int64_t)alb_globaltimer();
        const int rows = (r1 - r) < R ? (r1 - r) : R;
        const uint8_t * nib = sh.ring[slot];
        const uint16_t * scl = reinterpret_cast<const uint16_t *>(sh.ring[slot] + (size_t)R * rb);
        for (int i = 0;; ++i) {
            int ra, rc;
            if (s.unit == 2) { ra = 2 * (warp + MK_CONSUMERS * i); rc = ra + 1; }
            else { ra = warp + 2 * MK_CONSUMERS * i; rc = ra + MK_CONSUMERS; }
            if (ra >= rows) break;
            const int row = half ? rc : ra;
            const bool live = row < rows;
            const int rr = live ? row : ra;
            const uint8_t * nr = nib + (size_t)rr * rb;
            const uint16_t * sr = scl + (size_t)rr * sp;
            double a = 0.0;
#pragma unroll
            for (int k = 0; k < MK_RECS_H; ++k) {
                const int b = hl + 16 * k;
                if (b < nb) mk_dot(a, nr, sr, b, rlo[k], rhi[k], rsum[k], rdx[k]);
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (s.unit == 2) {
                const double up = __shfl_sync(0xffffffffu, a, 16);
                if (lane == 0) mk_emit(OUT, p, y, r + ra, a, up, add_res, &best_key);
            } else if (hl == 0 && live) {
                mk_emit(OUT, p, y, r + row, a, 0.0, add_res, &best_key);
            }
        }
        __syncwarp();
        if (lane == 0) alb_mbar_arrive(&sh.empty[slot]);
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g + 2] = (int64_t)alb_globaltimer();
    }
    if (OUT == 3) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long kk = __shfl_xor_sync(0xffffffffu, best_key, o);
            best_key = kk > best_key ? kk : best_key;
        }
        if (lane == 0) atomicMax(&sh.am, best_key);
    }
    return (int64_t)g;
}

// Returns the stage counter after the stream, or -1 on a timeout.  OUT == 3
// leaves the CTA's best (logit, index) key in sh.am.
__device__ __noinline__ int64_t mk_gemv(int OUT, const MkParams & p, MkShared & sh_arg, const MkStream s, uint32_t g, float * y,
                                        bool add_res) {
    MkShared & sh = mk_sh();
    (void)sh_arg;
    const MkPlan pl = mk_plan(s.K, s.unit);
    if (pl.P == 1) {
        switch (s.K) {
            case 32 * 16 * 5: return mk_gemv_hk<5>(OUT, p, s, g, y, add_res);
            case 32 * 16 * 4: return mk_gemv_hk<4>(OUT, p, s, g, y, add_res);
            case 32 * 16 * 2: return mk_gemv_hk<2>(OUT, p, s, g, y, add_res);
            default: break;
        }
        if (s.K <= 32 * 16 * MK_RECS_H) return mk_gemv_h(OUT, p, s, g, y, add_res);
    }
    unsigned long long best_key = 0ull;
    unsigned long long * best = &best_key;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int R = pl.R, P = pl.P;
    const int nb = (int)(s.K / 32);
    const int64_t rb = s.K / 2, sp = q4_scale_pitch(s.K);
    const int part = warp % P, uw = warp / P;
    const int b0 = nb * part / P, b1 = nb * (part + 1) / P;
    int4 rlo[MK_RECS], rhi[MK_RECS];
    int rsum[MK_RECS];
    double rdx[MK_RECS];
#pragma unroll
    for (int k = 0; k < MK_RECS; ++k) {
        const int b = b0 + lane + 32 * k;
        const int4 * rec = reinterpret_cast<const int4 *>(sh.u.xs + (b < b1 ? b : b0) * XREC_INTS);
        rlo[k] = rec[0];
        rhi[k] = rec[1];
        const int4 r2 = rec[2];
        rsum[k] = r2.y;
        rdx[k] = __hiloint2double(r2.w, r2.z);
    }
    int r0, r1;
    mk_range(s, r0, r1);
    int64_t * st_tr = (p.trace && blockIdx.x == 0 && threadIdx.x == 0) ? p.trace + 1024 : nullptr;
    for (int r = r0; r < r1; r += R, ++g) {
        const int slot = g % MK_NSLOT;
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g] = (int64_t)alb_globaltimer();
        if (!alb_mbar_wait(&sh.full[slot], (g / MK_NSLOT) & 1)) {
            if (lane == 0) atomicExch(p.err, ALB_DEVERR_MBAR_TIMEOUT);
            sh.abort_flag = 1;
            return -1;
        }
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g + 1] = (int64_t)alb_globaltimer();
        const int rows = (r1 - r) < R ? (r1 - r) : R;
        const uint8_t * nib = sh.ring[slot];
        const uint16_t * scl = reinterpret_cast<const uint16_t *>(sh.ring[slot] + (size_t)R * rb);
        if (P == 1) {
            // passes over row pairs: (2u, 2u + 1) for the gate/up units u = warp + 15 i,
            // else rows (warp + 30 i, warp + 30 i + 15)
            for (int i = 0;; ++i) {
                int ra, rc;
                if (s.unit == 2) { ra = 2 * (warp + MK_CONSUMERS * i); rc = ra + 1; }
                else { ra = warp + 2 * MK_CONSUMERS * i; rc = ra + MK_CONSUMERS; }
                if (ra >= rows) break;
                const bool has_c = rc < rows;
                const uint8_t * na = nib + (size_t)ra * rb, * nc = nib + (size_t)(has_c ? rc : ra) * rb;
                const uint16_t * sa = scl + (size_t)ra * sp, * sc = scl + (size_t)(has_c ? rc : ra) * sp;
                double aa = 0.0, ac = 0.0;
#pragma unroll
                for (int k = 0; k < MK_RECS; ++k) {
                    const int b = lane + 32 * k;
                    if (b < nb) {
                        mk_dot(aa, na, sa, b, rlo[k], rhi[k], rsum[k], rdx[k]);
                        if (has_c) mk_dot(ac, nc, sc, b, rlo[k], rhi[k], rsum[k], rdx[k]);
                    }
                }
                aa = alb_warp_sum_d(aa);
                if (has_c) ac = alb_warp_sum_d(ac);
                if (lane == 0) {
                    if (s.unit == 2) {
                        mk_emit(OUT, p, y, r + ra, aa, ac, add_res, best);
                    } else {
                        mk_emit(OUT, p, y, r + ra, aa, 0.0, add_res, best);
                        if (has_c) mk_emit(OUT, p, y, r + rc, ac, 0.0, add_res, best);
                    }
                }
            }
        } else {
            // unit uw, K part `part` of the warp; partials combined in shared memory
            const int n_units = rows / s.unit;
            if (uw < n_units) {
                const int rl = uw * s.unit;
                const uint8_t * na = nib + (size_t)rl * rb;
                const uint16_t * sa = scl + (size_t)rl * sp;
                double acc0 = 0.0, acc1 = 0.0;
#pragma unroll
                for (int k = 0; k < MK_RECS; ++k) {
                    const int b = b0 + lane + 32 * k;
                    if (b < b1) {
                        mk_dot(acc0, na, sa, b, rlo[k], rhi[k], rsum[k], rdx[k]);
                        if (s.unit == 2) mk_dot(acc1, na + rb, sa + sp, b, rlo[k], rhi[k], rsum[k], rdx[k]);
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
                mk_emit(OUT, p, y, r + warp * s.unit, a0, a1, add_res, best);
            }
            mk_bar();
        }
        __syncwarp();
        if (lane == 0) alb_mbar_arrive(&sh.empty[slot]);
        if (st_tr && 3 * g + 2 < 7168) st_tr[3 * g + 2] = (int64_t)alb_globaltimer();
    }
    if (OUT == 3) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long kk = __shfl_xor_sync(0xffffffffu, best_key, o);
            best_key = kk > best_key ? kk : best_key;
        }
        if ((threadIdx.x & 31) == 0) atomicMax(&sh.am, best_key);
    }
    return (int64_t)g;
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


// Attention of the new token, one (kv head h, cell split s) item per CTA
// (Hkv * S <= gridDim.x).  Same arithmetic as k_fa_scores / k_fa_pv:
//   QK-norm + RoPE of the G q heads (and of k, stored with v into the cache by
//   the split holding the new cell); scores s_c = fp32 fma chain over d in
//   order, times scale; split max -> the S CTAs of head h wait for one another
//   (bounded; all CTAs are co-resident under the cooperative launch) -> global
//   max M; p_c = v_expf(s_c - M); L and O = sum_c p_c V_c in double; the last
//   split (ticket) adds the S split records in split order and writes att.
// Cells [c0, c0 + 64) of the split come from shared memory (staged by
// mk_kv_stage during the QKV phase), the rest of a long split from L2/HBM.
static_assert(MK_MAX_G * 128 <= 2 * MK_CONSUMERS * 32, "two (g, d) outputs per thread");
static_assert(offsetof(MkAttSmem, kt) >= MK_STAGE_OFFSET, "staged inputs above the QKV records");
static_assert(MK_MAX_G * MK_ATT_MAX_CELLS <= 4 * MK_CONSUMERS * 32, "four numerators per thread");
static_assert(MK_MAX_G * MK_SC_PITCH * 4 <= sizeof(double) * MK_MAX_G * MK_ATT_MAX_CELLS, "scores fit the numerator array");
// merge scratch of one split: at most G*128/S + 1 outputs and 2 heads' L, each
// S doubles, i.e. <= (G*128 + 3 S) doubles, inside the numerator array (S <= 160)
static_assert((MK_MAX_G * 128 + 3 * 160) * 8 <= sizeof(double) * MK_MAX_G * MK_ATT_MAX_CELLS, "merge scratch fits");

__device__ __forceinline__ void mk_split(int n, int S, int s, int & c0, int & c1) {
    const int sz = (n + S - 1) / S;
    c0 = s * sz;
    c1 = min(n, c0 + sz);
    if (c0 > n) c0 = n;
}

// Lanes 1..31 of the producer warp, attention CTAs only: for every layer, once
// the consumers signal sh.stage_ok (the union's attention region is free: the
// previous layer's attention is over), copy the inputs of this CTA's
// attention that do not depend on the current token -- the cached K/V cells
// below pos (at most MK_KV_TILE), the layer's q/k norm weights and the RoPE row
// of pos -- into the union with 16-byte cp.async; each lane's completion
// arrives on sh.kvbar (expected count 31).  The region lies above the Q8_0
// records of the QKV phase, which the consumers write meanwhile.
__device__ void mk_stager(const MkParams & p, MkShared & sh_arg, int pos) {
    MkShared & sh = mk_sh();
    (void)sh_arg;
    const int lane = threadIdx.x & 31;
    const int h = blockIdx.x / p.S, s = blockIdx.x % p.S;
    int c0, c1;
    mk_split(pos + 1, p.S, s, c0, c1);
    int ce = min(c1, pos);
    ce = min(ce, c0 + MK_KV_TILE);
    const int ncp = ce > c0 ? ce - c0 : 0;
    MkAttSmem & A = sh.u.a;
    const int64_t row = (int64_t)p.Hkv * 128;
    const int total = ncp * 32 + 96;                    // 16-byte chunks
    for (int l = 0; l < p.n_layer; ++l) {
        if (!alb_mbar_wait_backoff(&sh.stage_ok, l & 1) || sh.abort_flag) break;
        const MkLayer & L = p.layers[l];
        for (int i = lane - 1; i < total; i += 31) {
            const void * src;
            void * dst;
            if (i < ncp * 32) {
                const int c = i >> 5, j = i & 15;
                const bool v = (i >> 4) & 1;
                src = (v ? L.vc : L.kc) + (size_t)(c0 + c) * row + (size_t)h * 128 + 8 * j;
                dst = v ? (void *)&A.vt[c][8 * j] : (void *)&A.kt[c][8 * j];
            } else {
                const int k = i - ncp * 32, j = k & 31;
                if (k < 32) { src = L.qn + 4 * j; dst = &A.qn[4 * j]; }
                else if (k < 64) { src = L.kn + 4 * j; dst = &A.kn[4 * j]; }
                else { src = reinterpret_cast<const float2 *>(p.rope) + (size_t)pos * 64 + 2 * j; dst = &A.rope[2 * j]; }
            }
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(alb_smem_addr(dst)), "l"(src) : "memory");
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" :: "r"(alb_smem_addr(&sh.kvbar)) : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");   // no copy in flight when the lane exits
}

// Barrier of the S CTAs of one kv head (same protocol as mk_grid_sync on the
// head's own count / generation words).
__device__ bool mk_group_sync(const MkParams & p, MkShared & sh_arg, unsigned * count, unsigned * gen, unsigned S) {
    MkShared & sh = mk_sh();
    (void)sh_arg;
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

// fp16 bits -> double bits of (value * 2^-1008) (see alb_h2d)
__device__ __forceinline__ double mk_vbits(uint32_t v) {
    return __hiloint2double((int)(((v & 0x7FFFu) << 10) | ((v & 0x8000u) << 16)), 0);
}

// Called after sh.kvbar completed for this layer.
template <int G>
__device__ __noinline__ bool mk_attention(const MkParams & p, MkShared & sh_arg, const MkLayer & L, int pos, int layer) {
    MkShared & sh = mk_sh();
    (void)sh_arg;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int item = blockIdx.x;
    int64_t * ct = (p.trace && tid == 0 && layer < 36 && gridDim.x <= 160)
                    ? p.trace + 8192 + (size_t)layer * 2 * gridDim.x + 2 * blockIdx.x : nullptr;
    if (ct) ct[0] = (int64_t)alb_globaltimer();
    if (item >= p.Hkv * p.S) return true;
    int64_t * ft = (p.trace && tid == 0 && layer < 36 && gridDim.x <= 160)
                    ? p.trace + 24576 + ((size_t)layer * gridDim.x + blockIdx.x) * 8 : nullptr;
    int64_t * fc = (p.trace && tid == 0 && item == 0 && layer < 36) ? p.trace + 20000 + layer * 16 : nullptr;
#define MK_FT(k) do { if (ft) ft[k] = (int64_t)alb_globaltimer(); if (fc) fc[k] = (int64_t)clock64(); } while (0)
#define MK_FC(k) do { if (fc) fc[k] = (int64_t)clock64(); } while (0)
    MK_FT(0);
    MkAttSmem & A = sh.u.a;
    const int n = pos + 1;
    const int64_t row = (int64_t)p.Hkv * 128;
    const int h = item / p.S, s = item % p.S;
    int c0, c1;
    mk_split(n, p.S, s, c0, c1);
    const int nc = c1 - c0;
    for (int g = warp; g < G; g += MK_CONSUMERS) {
        mk_norm_rope(p.qkv + (size_t)(h * G + g) * 128, A.qn, p.eps, A.rope, sh.qs[g], sh, g);
#pragma unroll
        for (int e = 0; e < 4; ++e) sh.qs[g][4 * lane + e] = __half2float(__float2half_rn(sh.qs[g][4 * lane + e]));
    }
    if (c0 < n && c1 == n && warp == MK_CONSUMERS - 1) {
        mk_norm_rope(p.qkv + (size_t)(p.Hq + h) * 128, A.kn, p.eps, A.rope, sh.ktmp, sh, 0);
        const bool in_tile = pos - c0 < MK_KV_TILE;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = 4 * lane + e;
            const uint16_t kh = alb_f2h(sh.ktmp[d]);
            const uint16_t vh = alb_f2h(p.qkv[(size_t)(p.Hq + p.Hkv + h) * 128 + d]);
            L.kc[(size_t)pos * row + h * 128 + d] = kh;
            L.vc[(size_t)pos * row + h * 128 + d] = vh;
            if (in_tile) { A.kt[pos - c0][d] = kh; A.vt[pos - c0][d] = vh; }
        }
    }
    mk_bar();   // q in smem; the new K/V cell is stored (visible to this CTA)
    MK_FT(6);
    // scores: thread (cell c, head g); fp32 fma chain over d = 0..127 in order
    float mx = -INFINITY;
    const int gl = tid % G;                           // G divides 32: fixed per lane
    for (int i = tid; i < nc * G; i += MK_CONSUMERS * 32) {
        const int c = c0 + i / G;
        const uint4 * kr = c - c0 < MK_KV_TILE ? reinterpret_cast<const uint4 *>(A.kt[c - c0])
                                               : reinterpret_cast<const uint4 *>(L.kc + (size_t)c * row + (size_t)h * 128);
        const float4 * q4 = reinterpret_cast<const float4 *>(sh.qs[gl]);
        float a = 0.0f;
#pragma unroll 4
        for (int j = 0; j < 16; ++j) {
            const uint4 kv = kr[j];
            const float4 qa = q4[2 * j], qb = q4[2 * j + 1];
            const float2 k0 = __half22float2(*reinterpret_cast<const __half2 *>(&kv.x));
            const float2 k1 = __half22float2(*reinterpret_cast<const __half2 *>(&kv.y));
            const float2 k2 = __half22float2(*reinterpret_cast<const __half2 *>(&kv.z));
            const float2 k3 = __half22float2(*reinterpret_cast<const __half2 *>(&kv.w));
            a = __fmaf_rn(k0.x, qa.x, a); a = __fmaf_rn(k0.y, qa.y, a);
            a = __fmaf_rn(k1.x, qa.z, a); a = __fmaf_rn(k1.y, qa.w, a);
            a = __fmaf_rn(k2.x, qb.x, a); a = __fmaf_rn(k2.y, qb.y, a);
            a = __fmaf_rn(k3.x, qb.z, a); a = __fmaf_rn(k3.y, qb.w, a);
        }
        const float v = __fmul_rn(a, p.scale);
        reinterpret_cast<float *>(A.pd)[gl * MK_SC_PITCH + (c - c0)] = v;
        mx = fmaxf(mx, v);
    }
    // max per head: lanes with equal lane % G hold the same head
#pragma unroll
    for (int o = 16; o >= G; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane < G) sh.red_f[warp][lane] = mx;
    mk_bar();
    if (tid < G) {
        float m = -INFINITY;
        for (int k = 0; k < MK_CONSUMERS; ++k) m = fmaxf(m, sh.red_f[k][tid]);
        __stcg(p.smax + ((size_t)h * p.S + s) * G + tid, m);
    }
    MK_FT(1);
    if (!mk_group_sync(p, sh, p.grp + 2 * h, p.grp + 2 * h + 1, (unsigned)p.S)) return false;
    MK_FT(2);
    if (warp == 0) {   // the S*G split maxima, loaded at once; lanes with equal lane % G hold one head
        float m = -INFINITY;
        for (int i = lane; i < p.S * G; i += 32) m = fmaxf(m, __ldcg(p.smax + (size_t)h * p.S * G + i));
#pragma unroll
        for (int o = 16; o >= G; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane < G) sh.red_f[0][lane] = m;
    }
    mk_bar();
    MK_FT(7);
    {
        float sv[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = tid + k * MK_CONSUMERS * 32;
            if (i < G * nc) sv[k] = reinterpret_cast<const float *>(A.pd)[(i / nc) * MK_SC_PITCH + i % nc];
        }
        mk_bar();   // every score read before the numerators overwrite them
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = tid + k * MK_CONSUMERS * 32;
            if (i < G * nc) {
                const int g = i / nc, c = i - g * nc;
                // p_c * 2^1008: exact, and p * (bits of v as a double) = p * v (alb_h2d)
                A.pd[g][c] = (double)alb_ref_expf(__fsub_rn(sv[k], sh.red_f[0][g])) * 0x1p1008;
            }
        }
    }
    mk_bar();
    MK_FT(3);
    // P.V: thread (g, d) owns output d of q head g (threads below G*128 - 480
    // own a second one); cells summed in double, four cells' loads at a time
    {
        double * rec = p.part + ((size_t)h * p.S + s) * G * 129;
        const int i0 = tid, i1 = tid + MK_CONSUMERS * 32;
        const bool two = i1 < G * 128;
        const int ga = i0 >> 7, da = i0 & 127;
        const int gb = two ? i1 >> 7 : ga, db = two ? i1 & 127 : da;
        const double * pa = A.pd[ga], * pb = A.pd[gb];
        double oa = 0.0, ob = 0.0;
        const int nt = min(nc, MK_KV_TILE);
        if (i0 < G * 128) {
            int c = 0;
            for (; c + 4 <= nt; c += 4) {
                uint32_t va[4], vb[4];
                double wa[4], wb[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    va[k] = A.vt[c + k][da]; wa[k] = pa[c + k];
                    vb[k] = A.vt[c + k][db]; wb[k] = pb[c + k];
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    oa = fma(wa[k], mk_vbits(va[k]), oa);
                    if (two) ob = fma(wb[k], mk_vbits(vb[k]), ob);
                }
            }
            for (; c < nt; ++c) {
                oa = fma(pa[c], mk_vbits(A.vt[c][da]), oa);
                if (two) ob = fma(pb[c], mk_vbits(A.vt[c][db]), ob);
            }
            for (; c < nc; ++c) {
                const uint16_t * vr = L.vc + (size_t)(c0 + c) * row + (size_t)h * 128;
                oa = fma(pa[c], mk_vbits(__ldcg(vr + da)), oa);
                if (two) ob = fma(pb[c], mk_vbits(__ldcg(vr + db)), ob);
            }
            MK_FC(8);
            __stcg(rec + ga * 129 + da, oa);
            if (two) __stcg(rec + gb * 129 + db, ob);
            MK_FC(9);
        }
        if (tid >= 32 && tid < 32 + G) {
            // L of head tid - 32 (these threads own a single output), four partial chains
            const int g = tid - 32;
            double l0 = 0.0, l1 = 0.0, l2 = 0.0, l3 = 0.0;
            int c = 0;
            for (; c + 4 <= nc; c += 4) { l0 += A.pd[g][c]; l1 += A.pd[g][c + 1]; l2 += A.pd[g][c + 2]; l3 += A.pd[g][c + 3]; }
            for (; c < nc; ++c) l0 += A.pd[g][c];
            __stcg(rec + g * 129 + 128, ((l0 + l1) + (l2 + l3)) * 0x1p-1008);
        }
    }
    MK_FT(4);
    // all S records of head h written -> split s merges outputs [o0, o1) of the
    // head's G*128, adding the split records in split order (all loads at once)
    if (!mk_group_sync(p, sh, p.grp + 2 * h, p.grp + 2 * h + 1, (unsigned)p.S)) return false;
    MK_FC(10);
    {
        const int S = p.S;
        const int o0 = G * 128 * s / S, o1 = G * 128 * (s + 1) / S, no = o1 - o0;
        const int g0 = o0 >> 7, ng = ((o1 - 1) >> 7) - g0 + 1;
        double * ov = A.pd[0];                          // [no][S] then [ng][S]
        double * lv = ov + no * S;
        const double * hb = p.part + (size_t)h * S * G * 129;
        for (int i = tid; i < (no + ng) * S; i += MK_CONSUMERS * 32) {
            const int r = i / S, k = i - r * S;
            double v;
            if (r < no) { const int o = o0 + r; v = __ldcg(hb + ((size_t)k * G + (o >> 7)) * 129 + (o & 127)); }
            else v = __ldcg(hb + ((size_t)k * G + g0 + (r - no)) * 129 + 128);
            (r < no ? ov[r * S + k] : lv[(r - no) * S + k]) = v;
        }
        mk_bar();
        MK_FC(11);
        for (int r = tid; r < no; r += MK_CONSUMERS * 32) {
            const int o = o0 + r, g = o >> 7;
            double Lt = 0.0, Ot = 0.0;
#pragma unroll 6
            for (int k = 0; k < S; ++k) { Lt += lv[(g - g0) * S + k]; Ot += ov[r * S + k]; }
            p.att[(size_t)(h * G + g) * 128 + (o & 127)] = Lt > 0.0 ? __double2float_rn(Ot / Lt) : 0.0f;
        }
    }
    MK_FT(5);
#undef MK_FT
#undef MK_FC
    if (ct) ct[1] = (int64_t)alb_globaltimer();
    return true;
}

// ------------------------------------------------------------ the kernel
template <int G>
__global__ void __launch_bounds__(MK_THREADS, 1)
k_decode_step(const __grid_constant__ MkParams p) {
    MkShared & sh = mk_sh();
    const int tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        for (int i = 0; i < MK_NSLOT; ++i) { alb_mbar_init(&sh.full[i], 1); alb_mbar_init(&sh.empty[i], MK_CONSUMERS); }
        alb_mbar_init(&sh.kvbar, 31);
        alb_mbar_init(&sh.stage_ok, 1);
        sh.abort_flag = 0;
        sh.am = 0ull;
        alb_mbar_fence_init();
    }
    __syncthreads();
    if (warp == MK_CONSUMERS) {
        if ((tid & 31) == 0) mk_producer(p, sh);
        else if ((int)blockIdx.x < p.Hkv * p.S) mk_stager(p, sh, p.pos[0]);
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
        for (int i = r0 + tid; i < r1; i += MK_CONSUMERS * 32) p.x[i] = mk_embed(p, token, i);
    }
    int64_t * tr = (p.trace && blockIdx.x == 0 && tid == 0) ? p.trace : nullptr;
    int tn = 0;
#define MK_TRACE() do { if (tr && tn < 1024) tr[tn++] = (int64_t)alb_globaltimer(); } while (0)
    MK_TRACE();
    const bool att_cta = (int)blockIdx.x < p.Hkv * p.S;
    for (int l = 0; l < p.n_layer && ok; ++l) {
        const MkLayer & L = p.layers[l];
        // the previous layer's attention is over: its staging region may be refilled
        if (att_cta && tid == 0) alb_mbar_arrive(&sh.stage_ok);
        // P1: attn norm + QKV
        if (l == 0) mk_quantize(p, nullptr, token, L.an, p.E, sh);
        else mk_quantize(p, p.x, 0, L.an, p.E, sh);
        MK_TRACE();
        { const int64_t gn = mk_gemv(0, p, sh, mk_stream(p, 4 * l + 0), g, p.qkv, false); ok = gn >= 0; g = (uint32_t)gn; }
        MK_TRACE();
        if (!ok || !mk_grid_sync(p, sh)) { ok = false; break; }
        MK_TRACE();
        // P2+P3: attention of the new token
        if (att_cta) {
            if (!alb_mbar_wait(&sh.kvbar, (uint32_t)(l & 1))) {
                if (tid == 0) atomicExch(p.err, ALB_DEVERR_MBAR_TIMEOUT);
                sh.abort_flag = 1;
                ok = false;
                break;
            }
        }
        if (!mk_attention<G>(p, sh, L, pos, l)) { ok = false; break; }
        MK_TRACE();
        MK_TRACE();
        MK_TRACE();
        if (!mk_grid_sync(p, sh)) { ok = false; break; }
        MK_TRACE();
        // P4: O projection + residual
        mk_quantize(p, p.att, 0, nullptr, p.Dq, sh);
        MK_TRACE();
        { const int64_t gn = mk_gemv(1, p, sh, mk_stream(p, 4 * l + 1), g, p.x, p.rank == 0); ok = gn >= 0; g = (uint32_t)gn; }
        MK_TRACE();
        if (!ok || !mk_grid_sync(p, sh)) { ok = false; break; }
        MK_TRACE();
        // P5: ffn norm + gate/up + SwiGLU
        mk_quantize(p, p.x, 0, L.fn, p.E, sh);
        MK_TRACE();
        { const int64_t gn = mk_gemv(2, p, sh, mk_stream(p, 4 * l + 2), g, p.h, false); ok = gn >= 0; g = (uint32_t)gn; }
        MK_TRACE();
        if (!ok || !mk_grid_sync(p, sh)) { ok = false; break; }
        MK_TRACE();
        // P6: down projection + residual
        mk_quantize(p, p.h, 0, nullptr, p.F, sh);
        MK_TRACE();
        { const int64_t gn = mk_gemv(1, p, sh, mk_stream(p, 4 * l + 3), g, p.x, p.rank == 0); ok = gn >= 0; g = (uint32_t)gn; }
        MK_TRACE();
        if (!ok || !mk_grid_sync(p, sh)) { ok = false; break; }
        MK_TRACE();
    }
    if (!ok) {
        sh.abort_flag = 1;   // the stager lanes stop at their next wait
        return;
    }
    // P7: output norm + lm head + argmax
    mk_quantize(p, p.x, 0, p.out_norm, p.E, sh);
    MK_TRACE();
    if (mk_gemv(3, p, sh, mk_stream(p, 4 * p.n_layer), g, p.logits, false) < 0) return;
    MK_TRACE();
#undef MK_TRACE
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
        int32_t nxt = 0x7FFFFFFF - (int32_t)(b & 0xFFFFFFFFu);
        if (b == 0ull || nxt < 0 || nxt >= p.v0 + p.V) {   // no logit was emitted: never feed an invalid row back
            atomicExch(p.err, ALB_DEVERR_BAD_TOKEN);
            nxt = 0;
        }
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
