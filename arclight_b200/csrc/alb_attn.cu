// Split-K flash attention over the fp16 KV cache (decode and multi-token split
// calls), sm_100a.
//
// Reference: nnml_compute_forward_flash_attn_ext_f16 (nnml/src/ops/arm/arm.cpp:
// 2196-2433), one sequence, causal: token t (position p0 + t) attends cells
// [0, p0 + t + 1); GQA broadcast of G = Hq/Hkv query heads per KV head.
//
// Semantics (the oracle's attention mode 0; independent of the split count):
// Q rounded to fp16 (arm.cpp:2307); score s_c = sequential fp32 fma chain over
// d of K.Q, times scale; M = max_c s_c; p_c = v_expf(s_c - M) (the reference's
// NEON exp, arm.cpp:1757-1787); L and every O_d in a canonical order: within
// each chunk of AT_CHUNK cells, cells in order in fp32 (L_c = L_c + p,
// O_c = fmaf(p, v, O_c)); the chunk sums widened to double and added in chunk
// order (in superchunks past AT_SUPER chunks); out = O / L.  These are the same
// operations on any GPU split.  Softmax is shift invariant: this is the
// reference's function with fp32/fp64 arithmetic in place of its fp16
// accumulators (within 1e-6 of an fp64 attention, while the reference's own
// fp16 rounding is 1e-3 .. 5e-2 from it).  fp32 chains inside a chunk keep the
// P.V on the fp32 pipe: B200 issues fp64 fmas at about a quarter of that rate.
//
// Two launches:
//   k_att_scores  CTA (kv head h, token t, split s): scores of the split's
//                 cells and its per-head maxima; for a decode step it first
//                 applies the per-head QK-RMSNorm and NEOX RoPE to the raw
//                 projection (qwen3.cpp:215-224, ops.cpp:830-938) and stores
//                 the new K/V cell (set_rows, ops.cpp:135-181);
//   k_att_pv      same grid: the global maxima, p, and per chunk the ordered
//                 sums (one thread per dimension, cells in order); the last
//                 CTA of (h, t) to finish adds the chunk partials in chunk
//                 order, writes the output and, for a decode step, the
//                 block_q8_0 records of the output (the O projection's input).
#include <cfloat>
#include <cmath>

#include "alb_common.cuh"
#include "alb_internal.h"
#include "alb_q4_dev.cuh"

namespace alb {

static constexpr int AT_CHUNK = 128;                    // canonical summation chunk (cells)
static constexpr int AT_ST = 64;                        // cells per staging step (AT_CHUNK / 2)
static constexpr int AT_NST = 3;                        // K ring depth of k_att_scores
static constexpr int AT_SST = 128;                      // cells per K stage of k_att_scores (one per thread)
static constexpr int AT_KPITCH = 272;                   // padded K row in shared memory
static constexpr size_t AT_SCORES_SMEM = (size_t)AT_NST * AT_SST * AT_KPITCH;   // 104,448 B

__device__ __forceinline__ void at_cp16(void * dst, const void * src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(alb_smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void at_cp4(void * dst, const void * src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(alb_smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void at_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void at_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// Chunks of n cells; superchunks of scn = ceil(chunks / AT_SUPER) consecutive
// chunks (one chunk each up to AT_SUPER chunks), at most AT_SUPER of them.
// The canonical sums add cells in order within a chunk, chunk sums in order
// within a superchunk and superchunk sums in order; a split holds whole
// superchunks, so its partials do not depend on the split count.
static constexpr int AT_SUPER = 64;
__host__ __device__ __forceinline__ int at_nchunks(int n) { return (n + AT_CHUNK - 1) / AT_CHUNK; }
__host__ __device__ __forceinline__ int at_scn(int nch) { return nch > AT_SUPER ? (nch + AT_SUPER - 1) / AT_SUPER : 1; }
__host__ __device__ __forceinline__ int at_nsuper(int nch) { const int k = at_scn(nch); return (nch + k - 1) / k; }
// Superchunk slots of one token's partials when it attends at most ncap cells:
// the most superchunks any n <= ncap has (64 chunks make 64 superchunks, 65 make 33).
__host__ __device__ __forceinline__ int at_nsuper_max(int ncap) {
    const int nch = at_nchunks(ncap);
    return nch < AT_SUPER ? nch : AT_SUPER;
}
__device__ __forceinline__ int at_splits_used(int n, int S) {
    const int ns = at_nsuper(at_nchunks(n));
    return ns < S ? ns : S;
}
// The chunk range [j0, j1) of split s of Su: superchunks [ns s / Su, ns (s + 1) / Su).
__device__ __forceinline__ void at_split(int nch, int Su, int s, int & j0, int & j1) {
    const int ns = at_nsuper(nch), k = at_scn(nch);
    j0 = (int)((int64_t)ns * s / Su) * k;
    j1 = min(nch, (int)((int64_t)ns * (s + 1) / Su) * k);
}

struct AttParams {
    const float * q = nullptr;        // [T][Hq][128] fp32 (when qkv is null)
    const float * qkv = nullptr;      // decode, fused: [Hq + 2 Hkv][128] raw projection of the token
    const float * qn = nullptr, * kn = nullptr;   // QK-norm weights [128]
    float eps = 1e-6f;
    const float2 * rope = nullptr;    // [max_pos][64] (cos, sin)
    const uint16_t * kc = nullptr;    // [cells][Hkv][128] fp16
    const uint16_t * vc = nullptr;
    uint16_t * kcw = nullptr, * vcw = nullptr;   // fused: where the new K/V cell goes (same caches)
    int Hq = 0, Hkv = 0, T = 1, S = 1, ncap = 0;
    int32_t pos0 = 0;
    const int32_t * pos_dev = nullptr;
    float scale = 0.0f;
    int * tickets = nullptr;          // [Hkv * T]
    float * smax = nullptr;           // [Hkv][T][S][G]
    float * scores = nullptr;         // [Hkv][T][G][ncap]
    double * part = nullptr;          // [Hkv][T][at_nsuper_max(ncap)][G][129]
    float * out = nullptr;            // [T][Hq][128]
    uint8_t * xq = nullptr;           // optional block_q8_0 records of out [T][Hq * 4]
    int * err = nullptr;              // device error word (bounded waits of the cluster kernel)
};

struct AtLayout { size_t tickets_off, smax_off, scores_off, part_off, bytes; };
static AtLayout at_layout(int Hq, int Hkv, int T, int S, int ncap) {
    const int G = Hq / Hkv;
    AtLayout l;
    l.tickets_off = 0;
    l.smax_off = ((size_t)Hkv * T * 4 + 255) & ~(size_t)255;
    l.scores_off = (l.smax_off + (size_t)Hkv * T * S * G * 4 + 255) & ~(size_t)255;
    l.part_off = (l.scores_off + (size_t)Hkv * T * G * ncap * 4 + 255) & ~(size_t)255;
    const size_t nsp = (size_t)at_nsuper_max(ncap);
    l.bytes = l.part_off + (size_t)Hkv * T * nsp * G * 129 * 8;
    return l;
}

// Per-head RMSNorm over 128 values * w, then NEOX RoPE at the position of cs,
// for NH heads at once (qwen3.cpp:215-224, ops.cpp:680-724, 830-938).  Thread d
// of 128 holds element d of head k in v[k] (heads k >= nh are idle).  Each
// head's mean is the reference's sequential double sum of the fp32 squares
// divided by 128: a parallel double sum stands in for it where the rounded
// float mean is certainly the same, one thread re-sums it sequentially where
// not.  Heads k < nq use wq, the others wk.  Returns the roped values in v.
// SUB: called by threads 0..127 of a larger CTA (named barrier 1 of 128
// threads instead of __syncthreads).
__device__ __forceinline__ void at_sync128(bool sub) {
    if (sub) asm volatile("bar.sync 1, 128;" ::: "memory");
    else __syncthreads();
}
template <int NH, bool SUB = false>
__device__ __forceinline__ void at_norm_rope_heads(float (&v)[NH], int nh, int nq, const float * __restrict__ wq,
                                                   const float * __restrict__ wk, float eps, float2 cs,
                                                   float (*hb)[128], double (*hred)[NH], double * hseq) {
    const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
    double part[NH];
#pragma unroll
    for (int k = 0; k < NH; ++k) {
        part[k] = (double)__fmul_rn(v[k], v[k]);
        hb[k][d] = v[k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int k = 0; k < NH; ++k) part[k] += __shfl_xor_sync(0xffffffffu, part[k], o);
    if (lane == 0)
#pragma unroll
        for (int k = 0; k < NH; ++k) hred[warp][k] = part[k];
    at_sync128(SUB);
    double tot[NH];
    bool sure[NH];
#pragma unroll
    for (int k = 0; k < NH; ++k) {
        tot[k] = ((hred[0][k] + hred[1][k]) + hred[2][k]) + hred[3][k];
        sure[k] = k >= nh || alb_rms_mean_certain(tot[k], 128);
    }
    if (d < nh && d < NH) {   // rare: the sequential sum of a head whose certificate failed
        bool mine_sure = true;
#pragma unroll
        for (int k = 0; k < NH; ++k) if (k == d) mine_sure = sure[k];
        if (!mine_sure) hseq[d] = alb_rms_seq_sum(hb[d], 128);
    }
    at_sync128(SUB);   // hseq ready; hb is rewritten below
#pragma unroll
    for (int k = 0; k < NH; ++k) {
        if (k >= nh) continue;
        const double sum = sure[k] ? tot[k] : hseq[k];
        const float mean = (float)(sum / 128.0);
        const float scale = 1.0f / sqrtf(__fadd_rn(mean, eps));
        hb[k][d] = __fmul_rn(__fmul_rn(v[k], scale), (k < nq ? wq : wk)[d]);
    }
    at_sync128(SUB);
#pragma unroll
    for (int k = 0; k < NH; ++k) {
        if (k >= nh) continue;
        if (d < 64) v[k] = __fsub_rn(__fmul_rn(hb[k][d], cs.x), __fmul_rn(hb[k][d + 64], cs.y));
        else        v[k] = __fadd_rn(__fmul_rn(hb[k][d - 64], cs.y), __fmul_rn(hb[k][d], cs.x));
    }
}

// --------------------------------------------------------------- scores
template <int G, bool FUSED>
__global__ void __launch_bounds__(128)
k_att_scores(const AttParams a) {
    extern __shared__ __align__(16) uint8_t at_ring[];   // AT_NST x AT_SST x AT_KPITCH
    __shared__ __align__(16) float qs[G][128];
    __shared__ __align__(16) float knew[128];
    __shared__ float hb[FUSED ? G + 1 : 1][128];
    __shared__ double hred[4][G + 1];
    __shared__ double hseq[G + 1];
    __shared__ float red[4][G];
    const int h = blockIdx.x, t = blockIdx.y, s = blockIdx.z, tid = threadIdx.x;
    // positions come from memory written before this graph replay started
    const int p0 = a.pos_dev ? a.pos_dev[0] : a.pos0;
    const int n = p0 + t + 1;
    const int Su = at_splits_used(n, a.S);
    if (s == 0 && tid == 0) a.tickets[h * a.T + t] = 0;   // re-armed for k_att_pv of this call
    if (s >= Su) return;
    int j0, j1;
    at_split(at_nchunks(n), Su, s, j0, j1);
    const int c0 = j0 * AT_CHUNK, c1 = min(n, j1 * AT_CHUNK);
    const int64_t row = (int64_t)a.Hkv * 128;
    const uint16_t * kb = a.kc + (size_t)h * 128;
    const int nst = (c1 - c0 + AT_SST - 1) / AT_SST;
    auto issue = [&](int i) {
        if (i < nst) {
            const int cb = c0 + i * AT_SST, rows = min(AT_SST, c1 - cb);
            uint8_t * dst = at_ring + (i % AT_NST) * AT_SST * AT_KPITCH;
            for (int p = tid; p < rows * 16; p += 128) {
                const int r = p >> 4, j = p & 15;
                at_cp16(dst + r * AT_KPITCH + j * 16, kb + (size_t)(cb + r) * row + j * 8);
            }
        }
        at_commit();   // one group per stage, empty past the end
    };
    // A decode step's cached cells were written by earlier steps: stream them
    // before waiting.  Other calls may follow the kernel that stored the cells.
    if constexpr (FUSED) {
#pragma unroll
        for (int i = 0; i < AT_NST - 1; ++i) issue(i);
    }
    alb_pdl_wait();
    if constexpr (!FUSED) {
#pragma unroll
        for (int i = 0; i < AT_NST - 1; ++i) issue(i);
    }
    if constexpr (FUSED) {
        // QK-norm + RoPE of this KV head's G query heads and, when this split
        // holds the new cell n - 1 (its last), of the new K, all heads at once,
        // from the raw projection of the token
        const float2 cs = a.rope[(size_t)(n - 1) * 64 + (tid & 63)];
        const bool with_k = c1 == n;
        float v[G + 1];
#pragma unroll
        for (int g = 0; g < G; ++g) v[g] = a.qkv[(size_t)(h * G + g) * 128 + tid];
        v[G] = with_k ? a.qkv[(size_t)(a.Hq + h) * 128 + tid] : 0.0f;
        at_norm_rope_heads<G + 1>(v, with_k ? G + 1 : G, G, a.qn, a.kn, a.eps, cs, hb, hred, hseq);
#pragma unroll
        for (int g = 0; g < G; ++g) qs[g][tid] = __half2float(__float2half_rn(v[g]));   // Q -> fp16 (arm.cpp:2307)
        if (with_k) {
            const uint16_t kh = alb_f2h(v[G]);
            knew[tid] = __half2float(__ushort_as_half(kh));
            a.kcw[(size_t)(n - 1) * row + (size_t)h * 128 + tid] = kh;
            a.vcw[(size_t)(n - 1) * row + (size_t)h * 128 + tid] =
                alb_f2h(a.qkv[(size_t)(a.Hq + a.Hkv + h) * 128 + tid]);
        }
    } else {
        for (int i = tid; i < G * 128; i += 128) {
            const int g = i / 128, d = i - g * 128;
            qs[g][d] = __half2float(__float2half_rn(a.q[((size_t)t * a.Hq + h * G + g) * 128 + d]));
        }
    }
    // thread tid: cell tid of each stage, all G heads (each K element is
    // converted once and feeds G independent chains)
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; ++g) mx[g] = -INFINITY;
    float * sc = a.scores + ((size_t)h * a.T + t) * G * a.ncap;
    for (int i = 0; i < nst; ++i) {
        at_wait<AT_NST - 2>();
        __syncthreads();   // stage i visible to all; stage i-1 consumed by all; q / knew visible
        issue(i + AT_NST - 1);
        const int c = c0 + i * AT_SST + tid;
        if (c < c1) {
            const uint8_t * kr = at_ring + (i % AT_NST) * AT_SST * AT_KPITCH + tid * AT_KPITCH;
            const bool knew_row = FUSED && c == n - 1;   // the new cell: its fp16 K from this kernel
            float acc[G];
#pragma unroll
            for (int g = 0; g < G; ++g) acc[g] = 0.0f;
#pragma unroll 4
            for (int j = 0; j < 16; ++j) {   // dims 8j .. 8j+7, in order (the reference's sequential chain)
                float kf[8];
                if (knew_row) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) kf[e] = knew[8 * j + e];
                } else {
                    const uint4 kv = *reinterpret_cast<const uint4 *>(kr + j * 16);
                    const uint32_t wd[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&wd[e]));
                        kf[2 * e] = f.x;
                        kf[2 * e + 1] = f.y;
                    }
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 qa = *reinterpret_cast<const float4 *>(&qs[g][8 * j]);
                    const float4 qb = *reinterpret_cast<const float4 *>(&qs[g][8 * j + 4]);
                    acc[g] = __fmaf_rn(kf[0], qa.x, acc[g]);
                    acc[g] = __fmaf_rn(kf[1], qa.y, acc[g]);
                    acc[g] = __fmaf_rn(kf[2], qa.z, acc[g]);
                    acc[g] = __fmaf_rn(kf[3], qa.w, acc[g]);
                    acc[g] = __fmaf_rn(kf[4], qb.x, acc[g]);
                    acc[g] = __fmaf_rn(kf[5], qb.y, acc[g]);
                    acc[g] = __fmaf_rn(kf[6], qb.z, acc[g]);
                    acc[g] = __fmaf_rn(kf[7], qb.w, acc[g]);
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float v = __fmul_rn(acc[g], a.scale);
                sc[(size_t)g * a.ncap + c] = v;
                mx[g] = fmaxf(mx[g], v);
            }
        }
    }
    at_wait<0>();
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float m = alb_warp_max(mx[g]);
        if (lane == 0) red[warp][g] = m;
    }
    __syncthreads();
    if (tid < G) {
        const int g = tid;
        a.smax[(((size_t)h * a.T + t) * a.S + s) * G + g] = fmaxf(fmaxf(red[0][g], red[1][g]), fmaxf(red[2][g], red[3][g]));
    }
    alb_pdl_trigger();
}

// --------------------------------------------------------------- P.V + merge
static constexpr int AT_PVR = 2;   // V / score stages in k_att_pv's ring (AT_PVR - 1 ahead; deeper rings measured slower)
template <int G>
__host__ __device__ constexpr size_t at_pv_stage() { return (size_t)AT_ST * 256 + (size_t)G * AT_ST * 4; }
template <int G>
__host__ __device__ constexpr size_t at_pv_smem() { return AT_PVR * at_pv_stage<G>() + (size_t)G * AT_ST * 8; }

// Lc + p[0] + p[stride] + ... + p[(n-1) stride] in order, in fp32 (a chunk's
// sum of p in the canonical order), the loads issued eight cells ahead of the
// dependent additions.
__device__ __forceinline__ float at_psum(float Lc, const float * p, int stride, int n) {
    int c = 0;
    for (; c + 8 <= n; c += 8) {
        float t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) t[u] = p[(c + u) * stride];
#pragma unroll
        for (int u = 0; u < 8; ++u) Lc = __fadd_rn(Lc, t[u]);
    }
    for (; c < n; ++c) Lc = __fadd_rn(Lc, p[c * stride]);
    return Lc;
}

static constexpr int AT_PV_THREADS = 160;   // warps 0-3: one thread per dimension; warp 4: the sums of p

// Ordered double sum of n values at p[0], p[stride], ... (n >= 0), loads issued
// eight at a time ahead of the additions.
__device__ __forceinline__ double at_ordered_sum(const double * __restrict__ p, size_t stride, int n) {
    double acc = 0.0;
    for (int j0 = 0; j0 < n; j0 += 8) {
        double t[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) t[k] = j0 + k < n ? __ldcg(p + (size_t)(j0 + k) * stride) : 0.0;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (j0 + k < n) acc += t[k];
    }
    return acc;
}

// out[g] = ordered double sum over k < n of p[k * G * 129 + g * 129] for every
// head g at once, loads issued eight partials (all heads) ahead.
template <int G>
__device__ __forceinline__ void at_ordered_sums(double (&out)[G], const double * __restrict__ p, int n) {
#pragma unroll
    for (int g = 0; g < G; ++g) out[g] = 0.0;
    for (int k0 = 0; k0 < n; k0 += 8) {
        double t[8][G];
#pragma unroll
        for (int k = 0; k < 8; ++k)
#pragma unroll
            for (int g = 0; g < G; ++g)
                t[k][g] = k0 + k < n ? __ldcg(p + (size_t)(k0 + k) * G * 129 + g * 129) : 0.0;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (k0 + k < n)
#pragma unroll
                for (int g = 0; g < G; ++g) out[g] += t[k][g];
    }
}

template <int G>
__global__ void __launch_bounds__(AT_PV_THREADS)
k_att_pv(const AttParams a) {
    extern __shared__ __align__(16) uint8_t at_sm[];   // 2 x (V rows [AT_ST][256 B] + scores [G][AT_ST]), p [G][AT_ST]
    float * pf = reinterpret_cast<float *>(at_sm + AT_PVR * at_pv_stage<G>());   // p of the step, [cell][head]
    __shared__ float Ms[G];
    __shared__ float redm[4][G];
    __shared__ double Ls[G];
    __shared__ int last_s;
    const int h = blockIdx.x, t = blockIdx.y, s = blockIdx.z, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int p0 = a.pos_dev ? a.pos_dev[0] : a.pos0;
    const int n = p0 + t + 1;
    const int Su = at_splits_used(n, a.S);
    if (s >= Su) return;
    const int nch = at_nchunks(n);
    int j0, j1;
    at_split(nch, Su, s, j0, j1);
    const int64_t row = (int64_t)a.Hkv * 128;
    const uint16_t * vb = a.vc + (size_t)h * 128;
    const float * sc = a.scores + ((size_t)h * a.T + t) * G * a.ncap;
    const size_t nspmax = (size_t)at_nsuper_max(a.ncap);
    double * part = a.part + ((size_t)h * a.T + t) * nspmax * G * 129;
    const int scn = at_scn(nch), nsp = at_nsuper(nch);
    double Osp[2][G];   // this superchunk's running sums (chunk sums in order)
    double Lsp = 0.0;
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int g = 0; g < G; ++g) Osp[e][g] = 0.0;
    // staging steps: AT_ST cells each, two per chunk, double-buffered
    const int cbeg = j0 * AT_CHUNK, cend = min(n, j1 * AT_CHUNK);
    const int nsteps = (cend - cbeg + AT_ST - 1) / AT_ST;
    // V rows of step i with cells in [lo, hi) and / or its scores
    auto issue_v = [&](int i, int lo, int hi) {
        const int cb = cbeg + i * AT_ST, rows = min(AT_ST, cend - cb);
        uint8_t * dst = at_sm + (i % AT_PVR) * at_pv_stage<G>();
        for (int p = tid; p < rows * 16; p += AT_PV_THREADS) {
            const int r = p >> 4, j = p & 15;
            if (cb + r >= lo && cb + r < hi) at_cp16(dst + r * 256 + j * 16, vb + (size_t)(cb + r) * row + j * 8);
        }
    };
    auto issue_s = [&](int i) {
        const int cb = cbeg + i * AT_ST, rows = min(AT_ST, cend - cb);
        float * sdst = reinterpret_cast<float *>(at_sm + (i % AT_PVR) * at_pv_stage<G>() + AT_ST * 256);
        for (int p = tid; p < rows * G; p += AT_PV_THREADS) {
            const int g = p / rows, c = p - g * rows;
            at_cp4(sdst + g * AT_ST + c, sc + (size_t)g * a.ncap + cb + c);
        }
    };
    // The cached cells' V (all but the new cell n - 1, which the score kernel of
    // a decode step stores) before waiting on the score kernel.
    const int n_old = a.qkv ? n - 1 : 0;   // fused decode call: cells < n - 1 are stable
#pragma unroll
    for (int k = 0; k < AT_PVR - 1; ++k) {
        if (k < nsteps) issue_v(k, 0, n_old);
        at_commit();
    }
    alb_pdl_wait();   // the scores, maxima (and the new V cell) come from k_att_scores
#pragma unroll
    for (int k = 0; k < AT_PVR - 1; ++k) {
        if (k < nsteps) {
            issue_v(k, n_old, n);
            issue_s(k);
        }
        at_commit();
    }
    {   // global maxima over the splits' maxima (max is exact: any order)
        float m = -INFINITY;
        if (tid < 128) {
            const int g = tid % G;
            const float * sm = a.smax + ((size_t)h * a.T + t) * a.S * G + g;
            for (int k = tid / G; k < Su; k += 128 / G) m = fmaxf(m, sm[(size_t)k * G]);
        }
#pragma unroll
        for (int o = G; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (tid < 128 && lane < G) redm[warp][lane] = m;
    }
    __syncthreads();
    if (tid < G) Ms[tid] = fmaxf(fmaxf(redm[0][tid], redm[1][tid]), fmaxf(redm[2][tid], redm[3][tid]));
    // O: threads t < 64 hold dimensions 2t, 2t + 1 of every head (one 32-bit V
    // load and one conversion per value serve G double fmas)
    float O[2][G];
    float Lc = 0.0f;   // warp 4, lane g < G: the chunk's sum of p for query head g
#pragma unroll
    for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int g = 0; g < G; ++g) O[e][g] = 0.0f;
    for (int i = 0; i < nsteps; ++i) {
        if (i + AT_PVR - 1 < nsteps) { issue_v(i + AT_PVR - 1, 0, n); issue_s(i + AT_PVR - 1); }
        at_commit();
        // commit groups: V of stages 0..R-2 (before the wait), then V + scores of
        // stages 0..R-2, then one per loop stage: stage i is complete when at
        // most R - 1 groups are pending
        at_wait<AT_PVR - 1>();
        __syncthreads();   // step i visible; Ms visible; pf free
        const uint8_t * stg = at_sm + (i % AT_PVR) * at_pv_stage<G>();
        const int cb = cbeg + i * AT_ST, rows = min(AT_ST, cend - cb);
        if (tid < AT_ST) {
            const float * ss = reinterpret_cast<const float *>(stg + AT_ST * 256);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float v = 0.0f;
                if (tid < rows) v = alb_ref_expf(__fsub_rn(ss[g * AT_ST + tid], Ms[g]));
                pf[tid * G + g] = v;
            }
        }
        __syncthreads();
        if (warp == 4) {
            if (lane < G) Lc = at_psum(Lc, pf + lane, G, rows);   // the chunk's sum of p, cells in order
        } else if (tid < 64) {
            // O_g,d = fmaf(p, v, O_g,d), cells in order (fp32, the canonical
            // within-chunk order).  Four cells per step with their loads issued first.
            const uint32_t * vs = reinterpret_cast<const uint32_t *>(stg) + tid;   // dims 2 tid, 2 tid + 1
            int c = 0;
            for (; c + 4 <= rows; c += 4) {
                float2 vf[4];
                float pp[4][G];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t w = vs[(c + u) * 64];
                    vf[u] = __half22float2(*reinterpret_cast<const __half2 *>(&w));
#pragma unroll
                    for (int g = 0; g < G; ++g) pp[u][g] = pf[(c + u) * G + g];
                }
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        O[0][g] = __fmaf_rn(pp[u][g], vf[u].x, O[0][g]);
                        O[1][g] = __fmaf_rn(pp[u][g], vf[u].y, O[1][g]);
                    }
            }
            for (; c < rows; ++c) {
                const uint32_t w = vs[c * 64];
                const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&w));
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float pg = pf[c * G + g];
                    O[0][g] = __fmaf_rn(pg, v.x, O[0][g]);
                    O[1][g] = __fmaf_rn(pg, v.y, O[1][g]);
                }
            }
        }
        // a chunk ends (every second step, or the split's last): its sums join
        // the superchunk's; a superchunk ends: its partial is written
        const int j = (cb - j0 * AT_CHUNK) / AT_CHUNK + j0;
        if ((i & 1) == 1 || i == nsteps - 1) {
            const bool send = (j + 1) % scn == 0 || j == nch - 1;
            double * pj = part + (size_t)(j / scn) * G * 129;
            if (tid < 64) {
#pragma unroll
                for (int e = 0; e < 2; ++e)
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        Osp[e][g] += (double)O[e][g];
                        O[e][g] = 0.0f;
                        if (send) { pj[g * 129 + 2 * tid + e] = Osp[e][g]; Osp[e][g] = 0.0; }
                    }
            } else if (warp == 4 && lane < G) {
                Lsp += (double)Lc;
                Lc = 0.0f;
                if (send) { pj[lane * 129 + 128] = Lsp; Lsp = 0.0; }
            }
        }
        __syncthreads();   // pf and buffer i & 1 consumed
    }
    at_wait<0>();
    // the last CTA of (h, t) adds every chunk's partial in chunk order
    __threadfence();
    __syncthreads();
    if (tid == 0) last_s = atomicAdd(&a.tickets[h * a.T + t], 1) == Su - 1;
    __syncthreads();
    if (!last_s) { alb_pdl_trigger(); return; }
    __threadfence();
    double Od[G];
    if (warp == 4) {
        if (lane < G) Ls[lane] = at_ordered_sum(part + lane * 129 + 128, (size_t)G * 129, nsp);
    } else {
        at_ordered_sums<G>(Od, part + tid, nsp);
    }
    __syncthreads();
    if (warp < 4) {
        float v[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            v[g] = Ls[g] > 0.0 ? __double2float_rn(Od[g] / Ls[g]) : 0.0f;
            a.out[((size_t)t * a.Hq + h * G + g) * 128 + tid] = v[g];
        }
        if (a.xq) {
            // quantize_row_q8_0 of the output (arm.cpp:1834-1851): warp w owns
            // block w of every head; the G reductions run interleaved
            float amax[G];
#pragma unroll
            for (int g = 0; g < G; ++g) amax[g] = fabsf(v[g]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int g = 0; g < G; ++g) amax[g] = fmaxf(amax[g], __shfl_xor_sync(0xffffffffu, amax[g], o));
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float d = amax[g] / 127.0f;
                const float id = d != 0.0f ? 1.0f / d : 0.0f;
                uint8_t * blk = a.xq + (((size_t)t * a.Hq + h * G + g) * 4 + warp) * 34;
                if (lane == 0) *reinterpret_cast<uint16_t *>(blk) = alb_f2h(d);
                blk[2 + lane] = (uint8_t)(int8_t)__float2int_rn(__fmul_rn(v[g], id));
            }
        }
    }
    if (tid == 0) a.tickets[h * a.T + t] = 0;
    alb_pdl_trigger();
}

// ------------------------------------------- decode: one cluster per KV head
// The decode step's attention of one token in ONE launch: a thread-block
// cluster of CL_CS CTAs per KV head, CTA r taking the contiguous chunks
// [nch r / CL_CS, nch (r + 1) / CL_CS) of the n = pos + 1 cells.  Same
// arithmetic and summation order as k_att_scores + k_att_pv (so the same
// results bit for bit):
//   1. QK-norm + RoPE of the G query heads (and, in the CTA holding cell
//      n - 1, of the new K, stored with the new V into the caches);
//   2. scores of the CTA's cells into shared memory, per-head maxima;
//   3. cluster barrier; the global maxima read from every CTA's shared memory
//      (DSMEM), so no workspace round trip and no second launch;
//   4. p, and per 128-cell chunk the ordered fp32 sums of p and p * v, kept in
//      shared memory (the K ring's region);
//   5. cluster barrier; each CTA merges whole 32-dimension output blocks
//      (chunk partials, read through DSMEM, added in double in chunk order),
//      writes them and their Q8_0 records; a last cluster barrier keeps every
//      CTA's partials alive until all reads are done.
// K and V stages of cached cells are streamed before the dependency wait.
// Every wait on a stage is bounded (error word set, results then invalid);
// every CTA takes both cluster barriers.  Cells per CTA <= CL_MAXC.
static constexpr int CL_CS = 8;                          // CTAs per cluster (portable size)
static constexpr int CL_ST = 64;                         // cells per stage
static constexpr int CL_KR = 2, CL_VR = 2;               // K / V ring stages
static constexpr int CL_MAXC = 1024;                     // cells per CTA (scores kept in shared memory)
static constexpr int CL_THREADS = 288;                   // warps 0-7: scores / P.V; warp 8: the sums of p

static_assert(CL_CS * CL_MAXC <= AT_SUPER * AT_CHUNK, "cluster path: one chunk per superchunk");

// The K ring's region holds the CTA's chunk partials (O and L of each head,
// [chunk][G][129] doubles) once the scores are done.
template <int G>
__host__ __device__ constexpr size_t cl_kregion() {
    return (size_t)CL_KR * CL_ST * AT_KPITCH > (size_t)(CL_MAXC / AT_CHUNK) * G * 129 * 8
               ? (size_t)CL_KR * CL_ST * AT_KPITCH : (size_t)(CL_MAXC / AT_CHUNK) * G * 129 * 8;
}
template <int G>
__host__ __device__ constexpr size_t cl_smem() {
    return cl_kregion<G>() + (size_t)CL_VR * CL_ST * 256 + (size_t)G * CL_MAXC * 4 +
           (size_t)G * CL_ST * 8 + 8 * (CL_KR + CL_VR);
}

__device__ __forceinline__ void cl_cp_arrive(uint64_t * bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" :: "r"(alb_smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void cl_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cl_map(const void * local, int rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(alb_smem_addr(local)), "r"(rank));
    return remote;
}
__device__ __forceinline__ double cl_ld_f64(uint32_t addr) {
    double v;
    asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ float cl_ld_remote(const float * local, int rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(alb_smem_addr(local)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

template <int G>
__global__ void __launch_bounds__(CL_THREADS, 1)
k_att_decode_cl(const AttParams a) {
    constexpr int GPT = G >= 4 ? G / 4 : 1;            // heads per thread in the score phase
    constexpr int GQ = G >= 4 ? 4 : G;                 // head groups of 64 threads there
    constexpr int HPT = G >= 2 ? G / 2 : 1;            // heads per thread in the P.V phase
    extern __shared__ __align__(16) uint8_t cl_sm[];
    uint8_t * kring = cl_sm;                                                     // [CL_KR][CL_ST][AT_KPITCH]
    uint8_t * vring = kring + cl_kregion<G>();                                   // [CL_VR][CL_ST][256]
    double * cpart = reinterpret_cast<double *>(kring);   // after the scores: [chunk - j0][G][129]
    float * sc = reinterpret_cast<float *>(vring + (size_t)CL_VR * CL_ST * 256); // [G][CL_MAXC]
    float * pf = reinterpret_cast<float *>(sc + (size_t)G * CL_MAXC);            // [G][CL_ST] p of the stage
    uint64_t * kfull = reinterpret_cast<uint64_t *>(pf + (size_t)2 * G * CL_ST);
    uint64_t * vfull = kfull + CL_KR;
    __shared__ __align__(16) unsigned short qh[G][128];   // fp16 bits of the rounded Q
    __shared__ __align__(16) unsigned short knewh[128];
    __shared__ __align__(16) uint16_t vnew[128];
    __shared__ float hb[G + 1][128];
    __shared__ double hred[4][G + 1];
    __shared__ double hseq[G + 1];
    __shared__ float cmax[G];
    __shared__ float redm[8][GPT];
    __shared__ float Ms[G];
    __shared__ int s_bad;
    const int r = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int p0 = a.pos_dev ? a.pos_dev[0] : a.pos0;    // written before this graph replay started
    const int n = p0 + 1;
    const int nch = at_nchunks(n);
    const int j0 = (int)((int64_t)nch * r / CL_CS), j1 = (int)((int64_t)nch * (r + 1) / CL_CS);
    const int c0 = j0 * AT_CHUNK, c1 = min(n, j1 * AT_CHUNK);
    const int ncell = c1 > c0 ? c1 - c0 : 0;
    const bool fits = ncell <= CL_MAXC;
    const int nst = fits ? (ncell + CL_ST - 1) / CL_ST : 0;
    const bool holder = ncell > 0 && c1 == n;            // this CTA holds the new cell n - 1
    const int64_t row = (int64_t)a.Hkv * 128;
    const uint16_t * kb = a.kc + (size_t)h * 128;
    const uint16_t * vb = a.vc + (size_t)h * 128;
    if (tid == 0) {
        for (int i = 0; i < CL_KR; ++i) alb_mbar_init(&kfull[i], CL_THREADS);
        for (int i = 0; i < CL_VR; ++i) alb_mbar_init(&vfull[i], CL_THREADS);
        s_bad = fits ? 0 : 1;
        alb_mbar_fence_init();
    }
    __syncthreads();
    // the O projection may launch now and stream its weights on the SMs' free
    // halves; it waits for this grid's completion before reading the output
    alb_pdl_trigger();
    // stage i of K (V): the cached rows by cp.async, completion counted on the
    // stage's mbarrier (one noinc arrival per thread); the new cell's row is
    // never copied (K: knew is used; V: vnew is written into the ring)
    auto issue = [&](bool is_v, int i, bool vnew_ready) {
        if (i >= nst) return;
        const int cb = c0 + i * CL_ST, rows = min(CL_ST, c1 - cb);
        uint8_t * dst = is_v ? vring + (size_t)(i % CL_VR) * CL_ST * 256
                             : kring + (size_t)(i % CL_KR) * CL_ST * AT_KPITCH;
        const int pitch = is_v ? 256 : AT_KPITCH;
        const uint16_t * src = is_v ? vb : kb;
        for (int p = tid; p < rows * 16; p += CL_THREADS) {
            const int rr = p >> 4, j = p & 15;
            if (cb + rr < n - 1) at_cp16(dst + rr * pitch + j * 16, src + (size_t)(cb + rr) * row + j * 8);
            else if (is_v && vnew_ready)
                *reinterpret_cast<uint4 *>(dst + rr * pitch + j * 16) = reinterpret_cast<const uint4 *>(vnew)[j];
        }
        cl_cp_arrive(is_v ? &vfull[i % CL_VR] : &kfull[i % CL_KR]);
    };
    for (int i = 0; i < CL_KR; ++i) issue(false, i, false);
    for (int i = 0; i < CL_VR; ++i) issue(true, i, false);
    // the norm weights and the RoPE row do not depend on the previous kernel
    const float2 cs = a.rope[(size_t)(n - 1) * 64 + (tid & 63)];
    alb_pdl_wait();

    // 1. QK-norm + RoPE (threads 0..127)
    if (tid < 128) {
        float v[G + 1];
#pragma unroll
        for (int g = 0; g < G; ++g) v[g] = a.qkv[(size_t)(h * G + g) * 128 + tid];
        v[G] = holder ? a.qkv[(size_t)(a.Hq + h) * 128 + tid] : 0.0f;
        const float vraw = holder ? a.qkv[(size_t)(a.Hq + a.Hkv + h) * 128 + tid] : 0.0f;
        at_norm_rope_heads<G + 1, true>(v, holder ? G + 1 : G, G, a.qn, a.kn, a.eps, cs, hb, hred, hseq);
#pragma unroll
        for (int g = 0; g < G; ++g) qh[g][tid] = __half_as_ushort(__float2half_rn(v[g]));   // Q -> fp16 (arm.cpp:2307)
        if (holder) {
            const uint16_t kh = alb_f2h(v[G]), vh = alb_f2h(vraw);
            knewh[tid] = kh;
            vnew[tid] = vh;
            a.kcw[(size_t)(n - 1) * row + (size_t)h * 128 + tid] = kh;
            a.vcw[(size_t)(n - 1) * row + (size_t)h * 128 + tid] = vh;
        }
    }
    __syncthreads();   // qh, knewh, vnew visible
    if (holder) {      // the new cell's V row, when its stage was issued above
        const int i = (n - 1 - c0) / CL_ST;
        if (i < CL_VR && tid < 16) {
            uint8_t * dst = vring + (size_t)(i % CL_VR) * CL_ST * 256 + (size_t)(n - 1 - c0 - i * CL_ST) * 256;
            reinterpret_cast<uint4 *>(dst)[tid] = reinterpret_cast<const uint4 *>(vnew)[tid];
        }
    }

    // 2. scores of the CTA's cells (thread: cell tid % 64 of the stage, heads
    //    GPT * (tid / 64) ..), the sequential fp32 chain over d
    const int cl = tid & (CL_ST - 1), gq = tid >> 6;
    const bool sthr = tid < 64 * GQ;
    float mx[GPT];
#pragma unroll
    for (int k = 0; k < GPT; ++k) mx[k] = -INFINITY;
    for (int i = 0; i < nst; ++i) {
        if (!alb_mbar_wait(&kfull[i % CL_KR], (uint32_t)((i / CL_KR) & 1))) {
            if (tid == 0) atomicExch(a.err, ALB_DEVERR_MBAR_TIMEOUT);
            s_bad = 1;
        }
        const int c = c0 + i * CL_ST + cl;
        if (sthr && c < c1) {
            const uint8_t * kr = kring + (size_t)(i % CL_KR) * CL_ST * AT_KPITCH + cl * AT_KPITCH;
            float acc[GPT];
#pragma unroll
            for (int k = 0; k < GPT; ++k) acc[k] = 0.0f;
#pragma unroll 4
            for (int j = 0; j < 16; ++j) {   // dims 8j .. 8j+7, in order (the reference's sequential chain)
                // acc = fma(f32(k_d), f32(q_d), acc) as one mixed-precision fma on the
                // fp16 bits (the product of two halves is exact in fp32)
                const uint4 kv = c == n - 1 ? *reinterpret_cast<const uint4 *>(knewh + 8 * j)
                                            : *reinterpret_cast<const uint4 *>(kr + j * 16);
                const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
                for (int k = 0; k < GPT; ++k) {
                    const uint4 qv = *reinterpret_cast<const uint4 *>(&qh[gq * GPT + k][8 * j]);
                    const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        acc[k] = alb_fma_f16_f32((unsigned short)(kw[e] & 0xFFFFu), (unsigned short)(qw[e] & 0xFFFFu), acc[k]);
                        acc[k] = alb_fma_f16_f32((unsigned short)(kw[e] >> 16), (unsigned short)(qw[e] >> 16), acc[k]);
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < GPT; ++k) {
                const float v = __fmul_rn(acc[k], a.scale);
                sc[(size_t)(gq * GPT + k) * CL_MAXC + (c - c0)] = v;
                mx[k] = fmaxf(mx[k], v);
            }
        }
        __syncthreads();   // K stage consumed by every thread
        issue(false, i + CL_KR, true);
    }
    // per-head maxima of this CTA: the 64 cells of a head group are warps 2gq, 2gq+1
#pragma unroll
    for (int k = 0; k < GPT; ++k) {
        const float m = alb_warp_max(mx[k]);
        if (lane == 0 && warp < 8) redm[warp][k] = m;
    }
    __syncthreads();
    if (tid < G) {
        const int q = tid / GPT, k = tid % GPT;
        cmax[tid] = fmaxf(redm[2 * q][k], redm[2 * q + 1][k]);
    }

    // 3. the global maxima: every CTA's cmax through distributed shared memory
    cl_barrier();
    if (tid < G) {
        float m = -INFINITY;
#pragma unroll
        for (int k = 0; k < CL_CS; ++k) m = fmaxf(m, cl_ld_remote(&cmax[tid], k));
        Ms[tid] = m;
    }
    __syncthreads();

    // 4. p, and per chunk the ordered fp32 sums (warps 0-7: O for dimension
    //    tid % 128 of heads (tid / 128) + 2k; warp 8: the sums of p)
    const int d = tid & 127, gh = (tid >> 7) & 1;
    float O[HPT];
    float Lc = 0.0f;
#pragma unroll
    for (int k = 0; k < HPT; ++k) O[k] = 0.0f;
    for (int i = 0; i < nst; ++i) {
        if (!alb_mbar_wait(&vfull[i % CL_VR], (uint32_t)((i / CL_VR) & 1))) {
            if (tid == 0) atomicExch(a.err, ALB_DEVERR_MBAR_TIMEOUT);
            s_bad = 1;
        }
        const int cb = c0 + i * CL_ST, rows = min(CL_ST, c1 - cb);
        if (tid < 64 * GQ) {
#pragma unroll
            for (int k = 0; k < GPT; ++k) {
                const int g = gq * GPT + k;
                float v = 0.0f;
                if (cl < rows) v = alb_ref_expf(__fsub_rn(sc[(size_t)g * CL_MAXC + (cb - c0) + cl], Ms[g]));
                pf[g * CL_ST + cl] = v;
            }
        }
        __syncthreads();
        if (warp == 8) {
            if (lane < G) Lc = at_psum(Lc, pf + lane * CL_ST, 1, rows);   // the chunk's sum of p, cells in order
        } else if (G >= 2 || gh == 0) {
            // O = fmaf(p, v, O), cells in order (fp32, the canonical within-chunk
            // order); four cells per step with their loads issued first
            const __half * vs = reinterpret_cast<const __half *>(vring + (size_t)(i % CL_VR) * CL_ST * 256) + d;
            int c = 0;
            for (; c + 4 <= rows; c += 4) {
                float vf[4], pp[4][HPT];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    vf[u] = __half2float(vs[(c + u) * 128]);
#pragma unroll
                    for (int k = 0; k < HPT; ++k) pp[u][k] = pf[(gh + 2 * k) * CL_ST + c + u];
                }
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int k = 0; k < HPT; ++k) O[k] = __fmaf_rn(pp[u][k], vf[u], O[k]);
            }
            for (; c < rows; ++c) {
                const float v = __half2float(vs[c * 128]);
#pragma unroll
                for (int k = 0; k < HPT; ++k) O[k] = __fmaf_rn(pf[(gh + 2 * k) * CL_ST + c], v, O[k]);
            }
        }
        const int j = j0 + (cb - c0) / AT_CHUNK;
        if ((i & 1) == 1 || i == nst - 1) {   // a chunk ends (two stages per chunk, or the CTA's last)
            double * pj = cpart + (size_t)(j - j0) * G * 129;
            if (warp == 8) {
                if (lane < G) { pj[lane * 129 + 128] = (double)Lc; Lc = 0.0f; }
            } else if (G >= 2 || gh == 0) {
#pragma unroll
                for (int k = 0; k < HPT; ++k) { pj[(gh + 2 * k) * 129 + d] = (double)O[k]; O[k] = 0.0f; }
            }
        }
        __syncthreads();   // V stage and pf consumed
        issue(true, i + CL_VR, true);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");   // no copy in flight past this point

    // 5. merge: this CTA's output blocks (head g, dims 32w .. 32w+31), block
    //    b = r, r + CL_CS, ... of the G * 4, one warp each.  Chunk j's partials
    //    are in the shared memory of the CTA that owns it (rank o with
    //    j0(o) <= j < j1(o)), read through distributed shared memory and added
    //    in chunk order (at_ordered_sum's order: 0.0 + P_0 + P_1 + ...).
    cl_barrier();   // every CTA's partials written (release / acquire at cluster scope)
    for (int b = r + CL_CS * warp; b < G * 4 && warp < 8; b += CL_CS * 8) {
        const int g = b >> 2, w = b & 3, dd = 32 * w + lane;
        double L = 0.0, Od = 0.0;
        int own = 0;
        for (int jb = 0; jb < nch; jb += 8) {
            double tl[8], to[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int j = jb + k;
                tl[k] = 0.0; to[k] = 0.0;
                if (j < nch) {
                    while (j >= (int)((int64_t)nch * (own + 1) / CL_CS)) ++own;
                    const int lj = j - (int)((int64_t)nch * own / CL_CS);
                    const uint32_t base = cl_map(cpart + ((size_t)lj * G + g) * 129, own);
                    tl[k] = cl_ld_f64(base + 128 * 8);
                    to[k] = cl_ld_f64(base + (uint32_t)dd * 8);
                }
            }
#pragma unroll
            for (int k = 0; k < 8; ++k)
                if (jb + k < nch) { L += tl[k]; Od += to[k]; }
        }
        const float v = L > 0.0 ? __double2float_rn(Od / L) : 0.0f;
        const int hq = h * G + g;
        a.out[(size_t)hq * 128 + dd] = v;
        if (a.xq) {   // quantize_row_q8_0 of the block (arm.cpp:1834-1851)
            int8_t q;
            uint16_t dh;
            q8_block_lane(v, q, dh);
            uint8_t * blk = a.xq + ((size_t)hq * 4 + w) * 34;
            if (lane == 0) *reinterpret_cast<uint16_t *>(blk) = dh;
            blk[2 + lane] = (uint8_t)q;
        }
    }
    if (s_bad && tid == 0 && !fits) atomicExch(a.err, ALB_DEVERR_MBAR_TIMEOUT);
    cl_barrier();   // no CTA leaves while another may still read its partials
}

template <int G>
static cudaError_t launch_att_cl_t(const AttParams & p, bool pdl, cudaStream_t st) {
    cudaError_t e = ensure_smem(k_att_decode_cl<G>, cl_smem<G>());
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL_CS, (unsigned)p.Hkv, 1);
    cfg.blockDim = dim3(CL_THREADS);
    cfg.dynamicSmemBytes = cl_smem<G>();
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL_CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, k_att_decode_cl<G>, p);
}

template <int G, bool FUSED>
static cudaError_t launch_att_t(const AttParams & p, bool pdl, cudaStream_t st) {
    cudaError_t e = ensure_smem(k_att_scores<G, FUSED>, AT_SCORES_SMEM);
    if (e == cudaSuccess) e = ensure_smem(k_att_pv<G>, at_pv_smem<G>());
    if (e != cudaSuccess) return e;
    const dim3 grid((unsigned)p.Hkv, (unsigned)p.T, (unsigned)p.S);
    e = alb_launch(k_att_scores<G, FUSED>, grid, dim3(128), AT_SCORES_SMEM, st, pdl, p);
    if (e != cudaSuccess) return e;
    return alb_launch(k_att_pv<G>, grid, dim3(AT_PV_THREADS), at_pv_smem<G>(), st, pdl, p);
}

template <bool FUSED>
static cudaError_t launch_att(const AttParams & p, bool pdl, cudaStream_t st) {
    if (p.Hkv <= 0 || p.Hq % p.Hkv != 0 || p.S < 1 || p.S > 65535 || p.T < 1 || p.T > 65535 || p.ncap <= 0)
        return cudaErrorInvalidValue;
    switch (p.Hq / p.Hkv) {
        case 1: return launch_att_t<1, FUSED>(p, pdl, st);
        case 2: return launch_att_t<2, FUSED>(p, pdl, st);
        case 4: return launch_att_t<4, FUSED>(p, pdl, st);
        case 8: return launch_att_t<8, FUSED>(p, pdl, st);
        default: return cudaErrorInvalidValue;
    }
}

static AttParams att_params(const FlashArgs & f) {
    AttParams p;
    const AtLayout l = at_layout(f.Hq, f.Hkv, f.T, f.S, f.ncap);
    uint8_t * ws = reinterpret_cast<uint8_t *>(f.ws);
    p.tickets = reinterpret_cast<int *>(ws + l.tickets_off);
    p.smax = reinterpret_cast<float *>(ws + l.smax_off);
    p.scores = reinterpret_cast<float *>(ws + l.scores_off);
    p.part = reinterpret_cast<double *>(ws + l.part_off);
    p.q = f.q; p.kc = f.kc; p.vc = f.vc; p.Hq = f.Hq; p.Hkv = f.Hkv; p.T = f.T; p.S = f.S; p.ncap = f.ncap;
    p.pos0 = f.pos0; p.pos_dev = f.pos_dev; p.scale = f.scale; p.out = f.out;
    p.xq = static_cast<uint8_t *>(f.xq);
    p.err = device_error_ptr();
    return p;
}

// Cells one decode-step cluster launch serves (the split kernels serve more).
int attn_decode_cluster_max_cells() { return CL_CS * CL_MAXC; }

size_t split_attn_ws_bytes(int Hq, int Hkv, int T, int S, int ncap) {
    return at_layout(Hq, Hkv, T, S, ncap).bytes;
}

cudaError_t launch_split_attn(const FlashArgs & f, cudaStream_t st) {
    if (!f.ws) return cudaErrorInvalidValue;
    return launch_att<false>(att_params(f), f.pdl, st);
}

cudaError_t launch_attn_decode(const FlashArgs & f, const QkvArgs & qa, bool cluster, cudaStream_t st) {
    if (!f.ws || f.T != 1 || !qa.qkv || !qa.rope || !qa.q_norm || !qa.k_norm) return cudaErrorInvalidValue;
    AttParams p = att_params(f);
    p.q = nullptr;
    p.qkv = qa.qkv; p.qn = qa.q_norm; p.kn = qa.k_norm; p.eps = qa.eps; p.rope = qa.rope;
    p.kcw = qa.kc; p.vcw = qa.vc;
    if (!p.err) return cudaErrorMemoryAllocation;
    if (!cluster) return launch_att<true>(p, f.pdl, st);
    if (p.Hkv <= 0 || p.Hq % p.Hkv != 0 || p.Hkv > 65535 || p.ncap > CL_CS * CL_MAXC) return cudaErrorInvalidValue;
    switch (p.Hq / p.Hkv) {
        case 1: return launch_att_cl_t<1>(p, f.pdl, st);
        case 2: return launch_att_cl_t<2>(p, f.pdl, st);
        case 4: return launch_att_cl_t<4>(p, f.pdl, st);
        case 8: return launch_att_cl_t<8>(p, f.pdl, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace alb
