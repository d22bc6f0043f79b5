/*
 * ArcLight hot-path ORACLE -- test infrastructure only (see oracle.h).
 *
 * CPU restatement of the reference's nnml arithmetic for the Qwen3 Q4_0
 * decode/prefill path.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs load this library, as the checker or
 * the timed CPU baseline; the CUDA product never calls it.
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared (oracle/Makefile).  Contraction
 * is off so every a*b+c below is two roundings unless written as fmaf().
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ fp16 */
/* ops.h:276-324 converts with round-to-nearest-even; _Float16 casts on x86-64
 * (GCC >= 12) are IEEE RNE conversions, bit-identical for all finite inputs. */
uint16_t orc_fp32_to_fp16(float f) {
    _Float16 h = (_Float16)f;
    uint16_t u;
    memcpy(&u, &h, 2);
    return u;
}

float orc_fp16_to_fp32(uint16_t u) {
    _Float16 h;
    memcpy(&h, &u, 2);
    return (float)h;
}

/* fp16 arithmetic as the ARMv8.2 FP16 vector unit does it (one rounding per
 * op).  double holds every product / sum of two fp16 values exactly. */
static inline uint16_t h_from_d(double d) { _Float16 h = (_Float16)d; uint16_t u; memcpy(&u, &h, 2); return u; }
static inline double   d_from_h(uint16_t u) { return (double)orc_fp16_to_fp32(u); }
static inline uint16_t h_add(uint16_t a, uint16_t b) { return h_from_d(d_from_h(a) + d_from_h(b)); }
static inline uint16_t h_mul(uint16_t a, uint16_t b) { return h_from_d(d_from_h(a) * d_from_h(b)); }
static inline uint16_t h_fma(uint16_t a, uint16_t b, uint16_t c) { return h_from_d(d_from_h(a) * d_from_h(b) + d_from_h(c)); }

float orc_neon_expf(float x);

/* ------------------------------------------------------- synthetic inputs */
uint64_t orc_splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* Inverse normal CDF by P. J. Acklam's rational approximation (2003), in
 * double, sampled at p_j = (j + 0.5) / 65537 and rounded to fp32.  The table is
 * the definition of the seeded "N(0,1)" stream; the product computes the same
 * table on the host and uploads it, so both sides draw identical values. */
static double acklam_inv_norm(double p) {
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
        double q = sqrt(-2.0 * log(p));
        return (((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
               ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1.0);
    }
    if (p <= phigh) {
        double q = p - 0.5, r = q * q;
        return (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q /
               (((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1.0);
    }
    double q = sqrt(-2.0 * log(1.0 - p));
    return -(((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
           ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1.0);
}

void orc_normal_table(float * t) {
    for (int j = 0; j <= 65536; ++j) t[j] = (float)acklam_inv_norm(((double)j + 0.5) / 65537.0);
}

float orc_normal(const float * t, uint64_t seed, uint64_t idx) {
    const uint64_t h = orc_splitmix64(seed + idx * 0xD1B54A32D192ED03ULL);
    const uint32_t i = (uint32_t)(h >> 48);
    const float frac = (float)((h >> 24) & 0xFFFFFFu) * (1.0f / 16777216.0f);
    const float lo = t[i], hi = t[i + 1];
    return fmaf(frac, hi - lo, lo);
}

uint64_t orc_tensor_seed(uint64_t model_seed, int layer, int kind) {
    return orc_splitmix64(model_seed * 0x100000001B3ULL + (uint64_t)((layer + 1) * 64 + kind));
}

/* ------------------------------------------------------------- quantizers */
/* quantize_row_q4_0_ref, types.cpp:352-378 */
void orc_quantize_row_q4_0(const float * x, orc_block_q4_0 * y, int64_t k) {
    const int64_t nb = k / ORC_QK;
    for (int64_t i = 0; i < nb; i++) {
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < ORC_QK; j++) {
            const float v = x[i * ORC_QK + j];
            if (amax < fabsf(v)) { amax = fabsf(v); max = v; }
        }
        const float d = max / -8;
        const float id = d ? 1.0f / d : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < ORC_QK / 2; ++j) {
            const float x0 = x[i * ORC_QK + j] * id;
            const float x1 = x[i * ORC_QK + ORC_QK / 2 + j] * id;
            const int8_t t0 = (int8_t)(x0 + 8.5f);
            const int8_t t1 = (int8_t)(x1 + 8.5f);
            const uint8_t xi0 = (uint8_t)(t0 < 15 ? t0 : 15);
            const uint8_t xi1 = (uint8_t)(t1 < 15 ? t1 : 15);
            y[i].qs[j] = (uint8_t)(xi0 | (xi1 << 4));
        }
    }
}

/* dequantize_row_q4_0, types.cpp:337-350 */
void orc_dequantize_row_q4_0(const orc_block_q4_0 * x, float * y, int64_t k) {
    const int64_t nb = k / ORC_QK;
    for (int64_t i = 0; i < nb; i++) {
        const float d = orc_fp16_to_fp32(x[i].d);
        for (int j = 0; j < ORC_QK / 2; ++j) {
            const int x0 = (x[i].qs[j] & 0x0F) - 8;
            const int x1 = (x[i].qs[j] >> 4) - 8;
            y[i * ORC_QK + j] = x0 * d;
            y[i * ORC_QK + j + ORC_QK / 2] = x1 * d;
        }
    }
}

/* vcvtnq_s32_f32: round to nearest, ties to even */
static inline int32_t cvt_rne(float v) { return (int32_t)nearbyintf(v); }

/* quantize_row_q8_0 NEON path, arm.cpp:1819-1853 (amax tree = exact max) */
void orc_quantize_row_q8_0(const float * x, orc_block_q8_0 * y, int64_t k) {
    const int64_t nb = k / ORC_QK;
    for (int64_t i = 0; i < nb; i++) {
        float amax = 0.0f;
        for (int j = 0; j < ORC_QK; j++) {
            const float a = fabsf(x[i * ORC_QK + j]);
            amax = a > amax ? a : amax;
        }
        const float d = amax / ((1 << 7) - 1);
        const float id = d ? 1.0f / d : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < ORC_QK; ++j) y[i].qs[j] = (int8_t)cvt_rne(x[i * ORC_QK + j] * id);
    }
}

/* quantize_row_q8_0_ref, types.cpp:494-514 (roundf: ties away from zero) */
void orc_quantize_row_q8_0_ref(const float * x, orc_block_q8_0 * y, int64_t k) {
    const int64_t nb = k / ORC_QK;
    for (int64_t i = 0; i < nb; i++) {
        float amax = 0.0f;
        for (int j = 0; j < ORC_QK; j++) {
            const float a = fabsf(x[i * ORC_QK + j]);
            amax = amax > a ? amax : a;
        }
        const float d = amax / ((1 << 7) - 1);
        const float id = d ? 1.0f / d : 0.0f;
        y[i].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < ORC_QK; ++j) y[i].qs[j] = (int8_t)roundf(x[i * ORC_QK + j] * id);
    }
}

/* dequantize_row_q8_0, types.cpp:483-492 */
void orc_dequantize_row_q8_0(const orc_block_q8_0 * x, float * y, int64_t k) {
    const int64_t nb = k / ORC_QK;
    for (int64_t i = 0; i < nb; i++) {
        const float d = orc_fp16_to_fp32(x[i].d);
        for (int j = 0; j < ORC_QK; ++j) y[i * ORC_QK + j] = x[i].qs[j] * d;
    }
}

/* make_block_q4_0x4 (types.cpp:133-166, interleave 4, XOR 0x88) driven by
 * repack_q4_0_to_q4_0_4_bl (types.cpp:168-197) */
int orc_repack_q4_0_4x4(const orc_block_q4_0 * src, orc_block_q4_0x4 * dst, int64_t nrow, int64_t k) {
    if (nrow % 4 != 0 || k % 8 != 0) return -1;
    const int64_t nb = k / ORC_QK;
    for (int64_t r = 0; r < nrow; r += 4) {
        for (int64_t x = 0; x < nb; x++) {
            orc_block_q4_0x4 out;
            for (int i = 0; i < 4; i++) out.d[i] = src[(r + i) * nb + x].d;
            for (int i = 0; i < 16; ++i) { /* end = QK4_0*2/4 = 16 chunks of 4 bytes */
                const int src_id = i % 4, src_off = (i / 4) * 4, dst_off = i * 4;
                uint32_t e;
                memcpy(&e, &src[(r + src_id) * nb + x].qs[src_off], 4);
                e ^= 0x88888888u;
                memcpy(&out.qs[dst_off], &e, 4);
            }
            *dst++ = out;
        }
    }
    return 0;
}

/* ---------------------------------------------------------------- threads */
typedef void (*orc_range_fn)(void * ctx, int64_t begin, int64_t end);
typedef struct { orc_range_fn fn; void * ctx; int64_t b, e; } orc_job;
static void * orc_job_run(void * p) { orc_job * j = (orc_job *)p; j->fn(j->ctx, j->b, j->e); return NULL; }

/* fn over [0, n) in n_threads contiguous ranges (one thread when n < min_n) */
static void orc_parallel_for_min(int n_threads, int64_t n, int64_t min_n, orc_range_fn fn, void * ctx) {
    if (n_threads <= 1 || n < min_n) { fn(ctx, 0, n); return; }
    if (n_threads > 64) n_threads = 64;
    if (n_threads > n) n_threads = (int)n;
    pthread_t th[64];
    orc_job jobs[64];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t].fn = fn; jobs[t].ctx = ctx;
        jobs[t].b = n * t / n_threads; jobs[t].e = n * (t + 1) / n_threads;
    }
    for (int t = 1; t < n_threads; ++t) pthread_create(&th[t], NULL, orc_job_run, &jobs[t]);
    orc_job_run(&jobs[0]);
    for (int t = 1; t < n_threads; ++t) pthread_join(th[t], NULL);
}

static void orc_parallel_for(int n_threads, int64_t n, orc_range_fn fn, void * ctx) {
    orc_parallel_for_min(n_threads, n, 64, fn, ctx);
}

/* ----------------------------------------------------------------- matvec */
static inline int32_t block_dot_q4_0_q8_0(const orc_block_q4_0 * w, const orc_block_q8_0 * a) {
    int32_t s = 0;
    for (int j = 0; j < 16; ++j) {
        s += ((w->qs[j] & 0x0F) - 8) * a->qs[j];
        s += ((w->qs[j] >> 4) - 8) * a->qs[j + 16];
    }
    return s;
}

typedef struct {
    const orc_block_q4_0 * W; const orc_block_q8_0 * xq; float * y; int32_t * dots; int64_t nb; int exact;
} gemv_ctx;

/* gemm.cpp:127-190: acc = vfmaq_f32(acc, vcvtq_n_f32_s32(16*I, 4), vmulq_f32(f32(ad), f32(bd)));
 * vcvtq_n_f32_s32(16*I, 4) == (float)I exactly (|16 I| < 2^24). */
static void gemv_range(void * p, int64_t r0, int64_t r1) {
    gemv_ctx * c = (gemv_ctx *)p;
    for (int64_t n = r0; n < r1; ++n) {
        const orc_block_q4_0 * w = c->W + n * c->nb;
        float acc = 0.0f;
        double accd = 0.0;
        for (int64_t b = 0; b < c->nb; ++b) {
            const int32_t I = block_dot_q4_0_q8_0(&w[b], &c->xq[b]);
            if (c->dots) c->dots[n * c->nb + b] = I;
            const float s = orc_fp16_to_fp32(c->xq[b].d) * orc_fp16_to_fp32(w[b].d);  /* exact: 11x11 bits */
            if (c->exact) accd += (double)I * (double)s;                               /* exact product */
            else acc = fmaf((float)I, s, acc);
        }
        c->y[n] = c->exact ? (float)accd : acc;
    }
}

void orc_gemv_q4_0_q8_0(const orc_block_q4_0 * W, const orc_block_q8_0 * xq, float * y,
                        int64_t N, int64_t K, int32_t * block_dots, int n_threads) {
    gemv_ctx c = { W, xq, y, block_dots, K / ORC_QK, 0 };
    orc_parallel_for(n_threads, N, gemv_range, &c);
}

/* The exactly rounded value of the same mat-vec: every block term I*dx*dw is
 * exact in double (38 significant bits); their double sum is exact whenever the
 * block scales of a row span < 2^7 (always, for these models), so the result
 * does not depend on the summation order.  It differs from the NEON fp32 chain
 * above by a few fp32 ulps. */
void orc_gemv_q4_0_q8_0_exact(const orc_block_q4_0 * W, const orc_block_q8_0 * xq, float * y,
                              int64_t N, int64_t K, int n_threads) {
    gemv_ctx c = { W, xq, y, NULL, K / ORC_QK, 1 };
    orc_parallel_for(n_threads, N, gemv_range, &c);
}

/* Tensor-parallel form of the exact mat-vec for the O / down projections
 * (model.cpp:21-54 split their input columns over the nodes): node j's partial
 * is the exactly rounded sum over its column slice of K/tp (32-aligned) and the
 * partials are added in node order in fp32, as GATHER does
 * (ops.cpp:1465-1511, nnml_vec_add_f32 arm.cpp:2435-2451). */
typedef struct { const orc_block_q4_0 * W; const orc_block_q8_0 * xq; float * y; int64_t nb; int tp; } gemv_tp_ctx;
static void gemv_tp_range(void * p, int64_t n0, int64_t n1) {
    const gemv_tp_ctx * c = (const gemv_tp_ctx *)p;
    const int64_t nbs = c->nb / c->tp;
    for (int64_t n = n0; n < n1; ++n) {
        const orc_block_q4_0 * w = c->W + n * c->nb;
        float acc = 0.0f;
        for (int j = 0; j < c->tp; ++j) {
            double accd = 0.0;
            for (int64_t b = j * nbs; b < (j + 1) * nbs; ++b) {
                const int32_t I = block_dot_q4_0_q8_0(&w[b], &c->xq[b]);
                const float s = orc_fp16_to_fp32(c->xq[b].d) * orc_fp16_to_fp32(w[b].d);
                accd += (double)I * (double)s;
            }
            acc = j == 0 ? (float)accd : acc + (float)accd;
        }
        c->y[n] = acc;
    }
}

void orc_gemv_q4_0_q8_0_exact_tp(const orc_block_q4_0 * W, const orc_block_q8_0 * xq, float * y,
                                 int64_t N, int64_t K, int tp, int n_threads) {
    gemv_tp_ctx c = { W, xq, y, K / ORC_QK, tp > 0 ? tp : 1 };
    orc_parallel_for(n_threads, N, gemv_tp_range, &c);
}

/* Tensor-parallel form of the NEON chain (the reference's own TP arithmetic):
 * node j runs nnml_gemv_q4_0_4x4_q8_0 (gemm.cpp:127-190) over its column slice
 * of K/tp (model.cpp:21-54 slices O / down by input columns in 32-aligned
 * units), a fresh fp32 fma chain from 0; GATHER then adds the node partials in
 * node order in fp32 (ops.cpp:1465-1511, nnml_vec_add_f32 arm.cpp:2435-2451). */
static void gemv_tp_chain_range(void * p, int64_t n0, int64_t n1) {
    const gemv_tp_ctx * c = (const gemv_tp_ctx *)p;
    const int64_t nbs = c->nb / c->tp;
    for (int64_t n = n0; n < n1; ++n) {
        const orc_block_q4_0 * w = c->W + n * c->nb;
        float acc = 0.0f;
        for (int j = 0; j < c->tp; ++j) {
            float part = 0.0f;
            for (int64_t b = j * nbs; b < (j + 1) * nbs; ++b) {
                const int32_t I = block_dot_q4_0_q8_0(&w[b], &c->xq[b]);
                const float s = orc_fp16_to_fp32(c->xq[b].d) * orc_fp16_to_fp32(w[b].d);
                part = fmaf((float)I, s, part);
            }
            acc = j == 0 ? part : acc + part;
        }
        c->y[n] = acc;
    }
}

void orc_gemv_q4_0_q8_0_tp(const orc_block_q4_0 * W, const orc_block_q8_0 * xq, float * y,
                           int64_t N, int64_t K, int tp, int n_threads) {
    gemv_tp_ctx c = { W, xq, y, K / ORC_QK, tp > 0 ? tp : 1 };
    orc_parallel_for(n_threads, N, gemv_tp_chain_range, &c);
}

/* nnml_vec_dot_q4_0_q8_0 NEON path (arm.cpp:633-692): blocks in pairs, two
 * float32x4 accumulators; lane i of vdotq_s32 sums elements 4i..4i+3 of the
 * low half and of the high half; vmlaq_n_f32 is contracted to fmla under
 * -ffp-contract=fast (CMakeLists.txt:11-20); vaddvq_f32 = (l0+l1)+(l2+l3). */
float orc_vec_dot_q4_0_q8_0(const orc_block_q4_0 * x, const orc_block_q8_0 * y, int64_t k) {
    const int64_t nb = k / ORC_QK;
    float sv0[4] = {0, 0, 0, 0}, sv1[4] = {0, 0, 0, 0};
    int64_t ib = 0;
    for (; ib + 1 < nb; ib += 2) {
        for (int h = 0; h < 2; ++h) {
            const orc_block_q4_0 * xb = &x[ib + h];
            const orc_block_q8_0 * yb = &y[ib + h];
            const float s = orc_fp16_to_fp32(xb->d) * orc_fp16_to_fp32(yb->d);
            float * sv = h ? sv1 : sv0;
            for (int l = 0; l < 4; ++l) {
                int32_t p = 0;
                for (int j = 0; j < 4; ++j) p += ((xb->qs[4 * l + j] & 0x0F) - 8) * yb->qs[4 * l + j];
                for (int j = 0; j < 4; ++j) p += ((xb->qs[4 * l + j] >> 4) - 8) * yb->qs[16 + 4 * l + j];
                sv[l] = fmaf((float)p, s, sv[l]);
            }
        }
    }
    float sumf = ((sv0[0] + sv0[1]) + (sv0[2] + sv0[3])) + ((sv1[0] + sv1[1]) + (sv1[2] + sv1[3]));
    for (; ib < nb; ++ib) { /* scalar tail, arm.cpp:675-691 */
        const int32_t sumi = block_dot_q4_0_q8_0(&x[ib], &y[ib]);
        sumf += sumi * orc_fp16_to_fp32(x[ib].d) * orc_fp16_to_fp32(y[ib].d);
    }
    return sumf;
}

typedef struct { const orc_block_q4_0 * W; const orc_block_q8_0 * xq; float * y; int64_t K; } mm_ctx;
static void mm_range(void * p, int64_t r0, int64_t r1) {
    mm_ctx * c = (mm_ctx *)p;
    const int64_t nb = c->K / ORC_QK;
    for (int64_t n = r0; n < r1; ++n) c->y[n] = orc_vec_dot_q4_0_q8_0(c->W + n * nb, c->xq, c->K);
}

/* forward_mul_mat_generic (common.cpp:120-248): one vec_dot per output row. */
void orc_mul_mat_generic(const orc_block_q4_0 * W, const orc_block_q8_0 * xq, float * y,
                         int64_t N, int64_t K, int n_threads) {
    mm_ctx c = { W, xq, y, K };
    orc_parallel_for(n_threads, N, mm_range, &c);
}

/* ------------------------------------------------------------ elementwise */
/* rms_norm_f32 (ops.cpp:680-724): double accumulation of float squares;
 * mean = (float)(sum / n); scale = 1/sqrtf(mean + eps); y = x*scale; then
 * the graph's MUL by the norm weight (binary.cpp:15-23, cgraph.cpp:115-120). */
void orc_rms_norm(const float * x, const float * w, float * y, int64_t rows, int64_t n, float eps) {
    for (int64_t r = 0; r < rows; ++r) {
        const float * xr = x + r * n;
        float * yr = y + r * n;
        double sum = 0.0;
        for (int64_t i = 0; i < n; ++i) sum += (double)(xr[i] * xr[i]);
        const float mean = (float)(sum / n);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int64_t i = 0; i < n; ++i) {
            const float v = xr[i] * scale;
            yr[i] = w ? v * w[i] : v;
        }
    }
}

/* nnml_rope_cache_init + rope_yarn (ops.cpp:747-771) with ext_factor = 0,
 * freq_scale = 1, mscale = attn_factor = 1, sin_sign = 1, no freq factors. */
void orc_rope_cache(int32_t pos, int64_t n_dims, float theta_scale, float * cache) {
    float theta = (float)pos;
    for (int64_t i0 = 0; i0 < n_dims; i0 += 2) {
        const float theta_interp = 1.0f * theta;
        cache[i0 + 0] = cosf(theta_interp) * 1.0f;
        cache[i0 + 1] = sinf(theta_interp) * 1.0f;
        theta *= theta_scale;
    }
}

/* rope_f32 NEOX branch (ops.cpp:830-938): pairs (ic, ic + n_dims/2). */
void orc_rope_neox(const float * x, float * y, int64_t n_heads, int64_t head_dim, int32_t pos, float freq_base) {
    const float theta_scale = powf(freq_base, -2.0f / (float)head_dim);
    float cache[1024];
    orc_rope_cache(pos, head_dim, theta_scale, cache);
    for (int64_t h = 0; h < n_heads; ++h) {
        const float * s = x + h * head_dim;
        float * d = y + h * head_dim;
        for (int64_t i0 = 0; i0 < head_dim; i0 += 2) {
            const int64_t ic = i0 / 2;
            const float c = cache[i0], sn = cache[i0 + 1];
            const float x0 = s[ic], x1 = s[ic + head_dim / 2];
            d[ic] = x0 * c - x1 * sn;
            d[ic + head_dim / 2] = x0 * sn + x1 * c;
        }
    }
}

static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* nnml_v_expf (arm.cpp:1757-1787), per lane: exp(x) = 2^n * (1 + poly(b)),
 * n = round(x/ln2) by the 1.5*2^23 shift, b = x - n*ln2 (two-part ln2), a
 * degree-5 polynomial; |n| > 126 / > 192 take the scaled and saturated paths.
 * vfmaq_f32(a, b, c) = a + b*c fused; vfmsq_f32(a, b, c) = a - b*c fused. */
float orc_neon_expf(float x) {
    const float r = 0x1.8p23f;
    const float z = fmaf(x, 0x1.715476p+0f, r);
    const float n = z - r;
    const float b = fmaf(-n, 0x1.7f7d1cp-20f, fmaf(-n, 0x1.62e4p-1f, x));
    const uint32_t e = f_bits(z) << 23;
    const float k = bits_f(e + f_bits(1.0f));
    const float u = b * b;
    const float j = fmaf(fmaf(fmaf(0x1.0e4020p-7f, b, 0x1.573e2ep-5f), u, fmaf(0x1.555e66p-3f, b, 0x1.fffdb6p-2f)), u,
                         0x1.ffffecp-1f * b);
    const float an = fabsf(n);
    if (!(an > 126.0f)) return fmaf(j, k, k);
    const uint32_t d = (n <= 0.0f) ? 0x82000000u : 0u;
    const float s1 = bits_f(d + 0x7f000000u);
    const float s2 = bits_f(e - d);
    if (an > 192.0f) return s1 * s1;
    return fmaf(s2, j, s2) * s1;
}

/* nnml_vec_swiglu_f32 NEON path (arm.cpp:1789-1809): silu(x) * g with x = gate,
 * g = up (nnml_swiglu_split(cur=gate, tmp=up), cgraph.cpp:610-614);
 * nnml_v_silu = x / (1 + v_expf(0 - x)). */
void orc_swiglu(const float * g, const float * u, float * y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        const float x = g[i];
        y[i] = (x / (1.0f + orc_neon_expf(0.0f - x))) * u[i];
    }
}

/* nnml_vec_add_f32 (arm.cpp:2435-2451): acc = src0; acc += src_j in order. */
void orc_gather_sum(const float * const * srcs, int n_srcs, float * dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        float acc = srcs[0][i];
        for (int j = 1; j < n_srcs; ++j) acc += srcs[j][i];
        dst[i] = acc;
    }
}

/* -------------------------------------------------------- flash attention */
/* nnml_vec_dot_f16 with FP16 vector arithmetic (arm.cpp:286-386, NEON branch):
 * 4 accumulators x 8 lanes, fp16 FMA; tree-reduce in fp16; last 8 lanes in fp32. */
static float vec_dot_f16_arm(int64_t n, const uint16_t * x, const uint16_t * y) {
    uint16_t sum[4][8];
    memset(sum, 0, sizeof(sum));
    const int64_t np = n & ~(int64_t)31;
    for (int64_t i = 0; i < np; i += 32)
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 8; ++l) sum[j][l] = h_fma(x[i + j * 8 + l], y[i + j * 8 + l], sum[j][l]);
    for (int l = 0; l < 8; ++l) { sum[0][l] = h_add(sum[0][l], sum[2][l]); sum[1][l] = h_add(sum[1][l], sum[3][l]); }
    for (int l = 0; l < 8; ++l) sum[0][l] = h_add(sum[0][l], sum[1][l]);
    float t[4];
    for (int l = 0; l < 4; ++l) t[l] = orc_fp16_to_fp32(sum[0][l]) + orc_fp16_to_fp32(sum[0][l + 4]);
    double sumf = (double)((t[0] + t[1]) + (t[2] + t[3]));
    for (int64_t i = np; i < n; ++i) sumf += (double)(orc_fp16_to_fp32(x[i]) * orc_fp16_to_fp32(y[i]));
    return (float)sumf;
}

/* nnml_compute_forward_flash_attn_ext_f16 (arm.cpp:2196-2433) for F16 K/V,
 * max_bias = 0, softcap = 0, no sinks; the mask admits cells [0, kv_len).
 *
 * mode 1 restates the reference's NEON loop: Q rounded to fp16, K.Q with
 * vec_dot_f16's fp16 FMA lanes, online softmax with libm expf, V accumulated
 * in fp16 (VKQ16), out = VKQ/S.
 * mode 0 is the fp32 semantics the CUDA kernels implement, defined so that it
 * does not depend on how the cells are split: Q rounded to fp16 (as the
 * reference), score s_c = (sequential fp32 fma chain over d of K.Q) * scale,
 * M = max_c s_c, p_c = v_expf(s_c - M) (nnml_v_expf, arm.cpp:1757-1787),
 * L = sum_c p_c and O_d = sum_c p_c V_cd summed in double, out_d = O_d / L.
 * Softmax is shift invariant, so this is the same function as the
 * reference's online form; only roundings differ. */
/* One (token, head) output of orc_flash_attn; the (token, head) pairs are
 * independent, so threads split them without changing any result. */
typedef struct {
    const float * q; const uint16_t * k, * v; const int32_t * kv_len;
    int64_t T, n_head, n_head_kv, D, nmax;
    float scale; int mode; float * out;
} fa_ctx;

static void fa_range(void * pc, int64_t b, int64_t e) {
    const fa_ctx * f = (const fa_ctx *)pc;
    const int64_t D = f->D, n_head = f->n_head;
    const int64_t rk2 = n_head / f->n_head_kv;
    const int64_t row = f->n_head_kv * D;
    const uint16_t * k = f->k, * v = f->v;
    const float scale = f->scale;
    uint16_t * Qh = (uint16_t *)malloc(D * 2);
    uint16_t * VKQ16 = (uint16_t *)malloc(D * 2);
    float * VKQ32 = (float *)malloc(D * 4);
    float * Qf = (float *)malloc(D * 4);
    float * sc = (float *)malloc(f->nmax * 4);
    double * Od = (double *)malloc((3 * D + (f->mode == 2 ? f->nmax : 0)) * sizeof(double));
    for (int64_t idx = b; idx < e; ++idx) {
        const int64_t t = idx / n_head, h = idx - t * n_head;
        const int64_t n_kv = f->kv_len[t];
        {
            const int64_t hk = h / rk2;
            const float * pq = f->q + (t * n_head + h) * D;
            float * po = f->out + (t * n_head + h) * D;
            for (int64_t d = 0; d < D; ++d) { Qh[d] = orc_fp32_to_fp16(pq[d]); Qf[d] = orc_fp16_to_fp32(Qh[d]); }
            if (f->mode == 2) {
                /* fp64 reference attention on the same inputs (fp16-rounded q, fp16
                 * K/V): scores, exp and sums in double, one rounding at the end;
                 * the yardstick for the errors of modes 0 and 1 */
                double M = -INFINITY;
                double * sd = Od + 3 * D;   /* scratch of n_kv doubles after Od, Oc and Os */
                for (int64_t c = 0; c < n_kv; ++c) {
                    const uint16_t * kc = k + c * row + hk * D;
                    double a = 0.0;
                    for (int64_t d = 0; d < D; ++d) a += (double)orc_fp16_to_fp32(kc[d]) * (double)Qf[d];
                    sd[c] = a * (double)scale;
                    M = sd[c] > M ? sd[c] : M;
                }
                double L = 0.0;
                for (int64_t d = 0; d < D; ++d) Od[d] = 0.0;
                for (int64_t c = 0; c < n_kv; ++c) {
                    const double p = exp(sd[c] - M);
                    const uint16_t * vc = v + c * row + hk * D;
                    L += p;
                    for (int64_t d = 0; d < D; ++d) Od[d] += p * (double)orc_fp16_to_fp32(vc[d]);
                }
                for (int64_t d = 0; d < D; ++d) po[d] = L > 0.0 ? (float)(Od[d] / L) : 0.0f;
                continue;
            }
            if (f->mode == 0) {
                float M = -INFINITY;
                for (int64_t c = 0; c < n_kv; ++c) {
                    const uint16_t * kc = k + c * row + hk * D;
                    float a = 0.0f;
                    for (int64_t d = 0; d < D; ++d) a = fmaf(orc_fp16_to_fp32(kc[d]), Qf[d], a);
                    sc[c] = a * scale;
                    M = sc[c] > M ? sc[c] : M;
                }
                /* chunked canonical order: within each ORC_FA_CHUNK-cell chunk, cells
                 * in order from 0 in fp32 (L_c = L_c + p, O_c = fmaf(p, v, O_c)); the
                 * chunk sums, widened to double, added in chunk order from 0 within
                 * each superchunk of scn consecutive chunks (scn = 1 up to
                 * ORC_FA_SUPER chunks); superchunk sums added in order from 0 */
                const int64_t nch = (n_kv + ORC_FA_CHUNK - 1) / ORC_FA_CHUNK;
                const int64_t scn = nch > ORC_FA_SUPER ? (nch + ORC_FA_SUPER - 1) / ORC_FA_SUPER : 1;
                double L = 0.0, Ls = 0.0;
                double * Os = Od + 2 * D;
                for (int64_t d = 0; d < D; ++d) { Od[d] = 0.0; Os[d] = 0.0; }
                for (int64_t j = 0; j < nch; ++j) {
                    const int64_t c0 = j * ORC_FA_CHUNK;
                    const int64_t c1 = c0 + ORC_FA_CHUNK < n_kv ? c0 + ORC_FA_CHUNK : n_kv;
                    float Lc = 0.0f;
                    float * Ocf = VKQ32;
                    for (int64_t d = 0; d < D; ++d) Ocf[d] = 0.0f;
                    for (int64_t c = c0; c < c1; ++c) {
                        const float p = orc_neon_expf(sc[c] - M);
                        const uint16_t * vc = v + c * row + hk * D;
                        Lc = Lc + p;
                        for (int64_t d = 0; d < D; ++d) Ocf[d] = fmaf(p, orc_fp16_to_fp32(vc[d]), Ocf[d]);
                    }
                    Ls += (double)Lc;
                    for (int64_t d = 0; d < D; ++d) Os[d] += (double)Ocf[d];
                    if ((j + 1) % scn == 0 || j == nch - 1) {   /* a superchunk ends */
                        L += Ls;
                        Ls = 0.0;
                        for (int64_t d = 0; d < D; ++d) { Od[d] += Os[d]; Os[d] = 0.0; }
                    }
                }
                for (int64_t d = 0; d < D; ++d) po[d] = L > 0.0 ? (float)(Od[d] / L) : 0.0f;
                continue;
            }
            float S = 0.0f, M = -INFINITY;
            memset(VKQ16, 0, D * 2);
            for (int64_t c = 0; c < n_kv; ++c) {
                const uint16_t * kc = k + c * row + hk * D;
                const uint16_t * vc = v + c * row + hk * D;
                float s = vec_dot_f16_arm(D, kc, Qh);
                s = s * scale;
                s += 0.0f; /* mask value of an admitted cell */
                const float Mold = M;
                float ms = 1.0f, vs = 1.0f;
                if (s > M) {
                    M = s;
                    ms = expf(Mold - M);
                    const uint16_t hm = orc_fp32_to_fp16(ms);
                    for (int64_t d = 0; d < D; ++d) VKQ16[d] = h_mul(VKQ16[d], hm);
                } else {
                    vs = expf(s - M);
                }
                const uint16_t hv = orc_fp32_to_fp16(vs);
                for (int64_t d = 0; d < D; ++d) VKQ16[d] = h_fma(vc[d], hv, VKQ16[d]);
                S = S * ms + vs;
            }
            for (int64_t d = 0; d < D; ++d) VKQ32[d] = orc_fp16_to_fp32(VKQ16[d]);
            const float S_inv = S > 0.0f ? 1.0f / S : 0.0f;
            for (int64_t d = 0; d < D; ++d) po[d] = VKQ32[d] * S_inv;
        }
    }
    free(Qh); free(VKQ16); free(VKQ32); free(Qf); free(sc); free(Od);
}

void orc_flash_attn_mt(const float * q, const uint16_t * k, const uint16_t * v, const int32_t * kv_len,
                       int64_t T, int64_t n_head, int64_t n_head_kv, int64_t D, float scale,
                       int mode, float * out, int n_threads) {
    int64_t nmax = 1;
    for (int64_t t = 0; t < T; ++t) nmax = kv_len[t] > nmax ? kv_len[t] : nmax;
    fa_ctx f = { q, k, v, kv_len, T, n_head, n_head_kv, D, nmax, scale, mode, out };
    orc_parallel_for_min(n_threads, T * n_head, 2, fa_range, &f);
}

void orc_flash_attn(const float * q, const uint16_t * k, const uint16_t * v, const int32_t * kv_len,
                    int64_t T, int64_t n_head, int64_t n_head_kv, int64_t D, float scale,
                    int mode, float * out) {
    orc_flash_attn_mt(q, k, v, kv_len, T, n_head, n_head_kv, D, scale, mode, out, 1);
}

/* ------------------------------------------------------------ Qwen3 model */
typedef struct {
    orc_block_q4_0 * wq, * wk, * wv, * wo, * wgate, * wup, * wdown;
    float * attn_norm, * ffn_norm, * q_norm, * k_norm;
    uint16_t * kc, * vc; /* [max_ctx][n_head_kv*head_dim] fp16 */
} orc_layer;

struct orc_model {
    orc_qwen3_config c;
    int32_t max_ctx, n_threads;
    orc_block_q4_0 * tok_embd, * output; /* output == tok_embd when tied */
    float * output_norm;
    orc_layer * layers;
    float * table;
    uint64_t seed;
    int exact;   /* 0: the reference's NEON fp32 chains (default); 1: exactly rounded mat-vecs */
    int tp;      /* > 1: O / down as tp column-slice partials added in node order */
};

typedef struct { const float * table; uint64_t seed; int64_t K; orc_block_q4_0 * dst; } gen_ctx;
static void gen_rows(void * p, int64_t r0, int64_t r1) {
    gen_ctx * g = (gen_ctx *)p;
    float * row = (float *)malloc(g->K * sizeof(float));
    for (int64_t r = r0; r < r1; ++r) {
        for (int64_t c = 0; c < g->K; ++c) row[c] = 0.02f * orc_normal(g->table, g->seed, (uint64_t)(r * g->K + c));
        orc_quantize_row_q4_0(row, g->dst + r * (g->K / ORC_QK), g->K);
    }
    free(row);
}

static orc_block_q4_0 * gen_q4(orc_model * m, int layer, int kind, int64_t rows, int64_t cols) {
    orc_block_q4_0 * w = (orc_block_q4_0 *)malloc((size_t)rows * (cols / ORC_QK) * sizeof(orc_block_q4_0));
    gen_ctx g = { m->table, orc_tensor_seed(m->seed, layer, kind), cols, w };
    orc_parallel_for(m->n_threads, rows, gen_rows, &g);
    return w;
}

static float * gen_norm(orc_model * m, int layer, int kind, int64_t n) {
    float * w = (float *)malloc(n * sizeof(float));
    const uint64_t seed = orc_tensor_seed(m->seed, layer, kind);
    for (int64_t i = 0; i < n; ++i) w[i] = 1.0f + 0.01f * orc_normal(m->table, seed, (uint64_t)i);
    return w;
}

orc_model * orc_model_create(const orc_qwen3_config * cfg, uint64_t seed, int32_t max_ctx, int n_threads) {
    orc_model * m = (orc_model *)calloc(1, sizeof(orc_model));
    m->c = *cfg;
    m->max_ctx = max_ctx;
    m->n_threads = n_threads > 0 ? n_threads : 1;
    m->seed = seed;
    m->exact = 0;
    m->tp = 1;
    m->table = (float *)malloc(65537 * sizeof(float));
    orc_normal_table(m->table);
    const orc_qwen3_config * c = &m->c;
    const int64_t E = c->n_embd, Dq = (int64_t)c->n_head * c->head_dim, Dkv = (int64_t)c->n_head_kv * c->head_dim;
    m->tok_embd = gen_q4(m, -1, ORC_T_TOK_EMBD, c->n_vocab, E);
    m->output = c->tied ? m->tok_embd : gen_q4(m, -1, ORC_T_OUTPUT, c->n_vocab, E);
    m->output_norm = gen_norm(m, -1, ORC_T_OUTPUT_NORM, E);
    m->layers = (orc_layer *)calloc(c->n_layer, sizeof(orc_layer));
    for (int l = 0; l < c->n_layer; ++l) {
        orc_layer * L = &m->layers[l];
        L->attn_norm = gen_norm(m, l, ORC_T_ATTN_NORM, E);
        L->wq = gen_q4(m, l, ORC_T_WQ, Dq, E);
        L->wk = gen_q4(m, l, ORC_T_WK, Dkv, E);
        L->wv = gen_q4(m, l, ORC_T_WV, Dkv, E);
        L->wo = gen_q4(m, l, ORC_T_WO, E, Dq);
        L->q_norm = gen_norm(m, l, ORC_T_Q_NORM, c->head_dim);
        L->k_norm = gen_norm(m, l, ORC_T_K_NORM, c->head_dim);
        L->ffn_norm = gen_norm(m, l, ORC_T_FFN_NORM, E);
        L->wgate = gen_q4(m, l, ORC_T_GATE, c->n_ff, E);
        L->wup = gen_q4(m, l, ORC_T_UP, c->n_ff, E);
        L->wdown = gen_q4(m, l, ORC_T_DOWN, E, c->n_ff);
        L->kc = (uint16_t *)calloc((size_t)max_ctx * Dkv, 2);
        L->vc = (uint16_t *)calloc((size_t)max_ctx * Dkv, 2);
    }
    return m;
}

void orc_model_free(orc_model * m) {
    if (!m) return;
    for (int l = 0; l < m->c.n_layer; ++l) {
        orc_layer * L = &m->layers[l];
        free(L->wq); free(L->wk); free(L->wv); free(L->wo); free(L->wgate); free(L->wup); free(L->wdown);
        free(L->attn_norm); free(L->ffn_norm); free(L->q_norm); free(L->k_norm); free(L->kc); free(L->vc);
    }
    free(m->layers);
    if (m->output != m->tok_embd) free(m->output);
    free(m->tok_embd);
    free(m->output_norm);
    free(m->table);
    free(m);
}

void orc_model_reset(orc_model * m) {
    const int64_t Dkv = (int64_t)m->c.n_head_kv * m->c.head_dim;
    for (int l = 0; l < m->c.n_layer; ++l) {
        memset(m->layers[l].kc, 0, (size_t)m->max_ctx * Dkv * 2);
        memset(m->layers[l].vc, 0, (size_t)m->max_ctx * Dkv * 2);
    }
}

typedef struct { orc_model * m; int64_t n; uint64_t seed; } fill_ctx;

static void fill_range(void * pc, int64_t b, int64_t e) {   /* layers [b, e) */
    const fill_ctx * f = (const fill_ctx *)pc;
    const int64_t Dkv = (int64_t)f->m->c.n_head_kv * f->m->c.head_dim;
    for (int64_t l = b; l < e; ++l) {
        const uint64_t sk = orc_tensor_seed(f->seed, (int)l, 62), sv = orc_tensor_seed(f->seed, (int)l, 63);
        for (int64_t i = 0; i < f->n * Dkv; ++i) {
            f->m->layers[l].kc[i] = orc_fp32_to_fp16(orc_normal(f->m->table, sk, (uint64_t)i));
            f->m->layers[l].vc[i] = orc_fp32_to_fp16(orc_normal(f->m->table, sv, (uint64_t)i));
        }
    }
}

void orc_model_fill_kv(orc_model * m, int32_t n_pos, uint64_t seed) {
    if (n_pos > m->max_ctx) n_pos = m->max_ctx;
    fill_ctx f = { m, n_pos, seed };
    orc_parallel_for_min(m->n_threads, m->c.n_layer, 2, fill_range, &f);
}

const orc_block_q4_0 * orc_model_q4_tensor(orc_model * m, int layer, int kind, int64_t * rows, int64_t * cols) {
    const orc_qwen3_config * c = &m->c;
    const int64_t E = c->n_embd, Dq = (int64_t)c->n_head * c->head_dim, Dkv = (int64_t)c->n_head_kv * c->head_dim;
    if (layer < 0) {
        if (kind == ORC_T_TOK_EMBD) { *rows = c->n_vocab; *cols = E; return m->tok_embd; }
        if (kind == ORC_T_OUTPUT)   { *rows = c->n_vocab; *cols = E; return m->output; }
        return NULL;
    }
    if (layer >= c->n_layer) return NULL;
    orc_layer * L = &m->layers[layer];
    switch (kind) {
        case ORC_T_WQ:   *rows = Dq;     *cols = E;      return L->wq;
        case ORC_T_WK:   *rows = Dkv;    *cols = E;      return L->wk;
        case ORC_T_WV:   *rows = Dkv;    *cols = E;      return L->wv;
        case ORC_T_WO:   *rows = E;      *cols = Dq;     return L->wo;
        case ORC_T_GATE: *rows = c->n_ff; *cols = E;     return L->wgate;
        case ORC_T_UP:   *rows = c->n_ff; *cols = E;     return L->wup;
        case ORC_T_DOWN: *rows = E;      *cols = c->n_ff; return L->wdown;
        default: return NULL;
    }
}

const float * orc_model_f32_tensor(orc_model * m, int layer, int kind, int64_t * n) {
    const orc_qwen3_config * c = &m->c;
    if (layer < 0) { if (kind == ORC_T_OUTPUT_NORM) { *n = c->n_embd; return m->output_norm; } return NULL; }
    if (layer >= c->n_layer) return NULL;
    orc_layer * L = &m->layers[layer];
    switch (kind) {
        case ORC_T_ATTN_NORM: *n = c->n_embd; return L->attn_norm;
        case ORC_T_FFN_NORM:  *n = c->n_embd; return L->ffn_norm;
        case ORC_T_Q_NORM:    *n = c->head_dim; return L->q_norm;
        case ORC_T_K_NORM:    *n = c->head_dim; return L->k_norm;
        default: return NULL;
    }
}

/* MUL_MAT over T rows: each row quantized to Q8_0 (arm.cpp:1886-1897), then the
 * repacked gemv/gemm per row (arm.cpp:1911-1925). */
static void matmul_rows(orc_model * m, const orc_block_q4_0 * W, const float * x, float * y,
                        int64_t T, int64_t N, int64_t K, orc_block_q8_0 * qbuf) {
    for (int64_t t = 0; t < T; ++t) {
        orc_quantize_row_q8_0(x + t * K, qbuf, K);
        if (m->exact) orc_gemv_q4_0_q8_0_exact(W, qbuf, y + t * N, N, K, m->n_threads);
        else orc_gemv_q4_0_q8_0(W, qbuf, y + t * N, N, K, NULL, m->n_threads);
    }
}

void orc_model_set_exact(orc_model * m, int exact) { m->exact = exact; }
void orc_model_set_tp(orc_model * m, int tp) { m->tp = tp > 0 ? tp : 1; }

/* O / down projections: tp > 1 forms the node partials over the column slices
 * and adds them in node order (the chain of each slice in the default mode,
 * exactly rounded slice sums in exact mode). */
static void matmul_rows_cols_split(orc_model * m, const orc_block_q4_0 * W, const float * x, float * y,
                                   int64_t T, int64_t N, int64_t K, orc_block_q8_0 * qbuf) {
    if (m->tp <= 1) { matmul_rows(m, W, x, y, T, N, K, qbuf); return; }
    for (int64_t t = 0; t < T; ++t) {
        orc_quantize_row_q8_0(x + t * K, qbuf, K);
        if (m->exact) orc_gemv_q4_0_q8_0_exact_tp(W, qbuf, y + t * N, N, K, m->tp, m->n_threads);
        else orc_gemv_q4_0_q8_0_tp(W, qbuf, y + t * N, N, K, m->tp, m->n_threads);
    }
}

int orc_model_forward(orc_model * m, const int32_t * tokens, int32_t T, int32_t pos0,
                      int fa_mode, float * logits, float * hidden) {
    const orc_qwen3_config * c = &m->c;
    if (T <= 0 || pos0 < 0 || pos0 + T > m->max_ctx) return -1;
    const int64_t E = c->n_embd, HD = c->head_dim, Dq = (int64_t)c->n_head * HD, Dkv = (int64_t)c->n_head_kv * HD;
    const int64_t Kmax = (E > Dq ? (E > c->n_ff ? E : c->n_ff) : (Dq > c->n_ff ? Dq : c->n_ff));
    float * x   = (float *)malloc(T * E * 4);
    float * h   = (float *)malloc(T * Kmax * 4);
    float * q   = (float *)malloc(T * Dq * 4);
    float * k   = (float *)malloc(T * Dkv * 4);
    float * v   = (float *)malloc(T * Dkv * 4);
    float * att = (float *)malloc(T * Dq * 4);
    float * g   = (float *)malloc(T * c->n_ff * 4);
    float * u   = (float *)malloc(T * c->n_ff * 4);
    float * o   = (float *)malloc(T * E * 4);
    int32_t * kv_len = (int32_t *)malloc(T * 4);
    orc_block_q8_0 * qb = (orc_block_q8_0 *)malloc((Kmax / ORC_QK) * sizeof(orc_block_q8_0));
    /* get_rows on tok_embd (ops.cpp:12-52) */
    for (int32_t t = 0; t < T; ++t) {
        if (tokens[t] < 0 || tokens[t] >= c->n_vocab) { T = 0; break; }
        orc_dequantize_row_q4_0(m->tok_embd + (int64_t)tokens[t] * (E / ORC_QK), x + t * E, E);
        kv_len[t] = pos0 + t + 1;
    }
    int rc = T > 0 ? 0 : -2;
    int64_t Tcur = T;
    for (int l = 0; rc == 0 && l < c->n_layer; ++l) {
        orc_layer * L = &m->layers[l];
        orc_rms_norm(x, L->attn_norm, h, Tcur, E, c->eps);
        matmul_rows(m, L->wq, h, q, Tcur, Dq, E, qb);
        matmul_rows(m, L->wk, h, k, Tcur, Dkv, E, qb);
        matmul_rows(m, L->wv, h, v, Tcur, Dkv, E, qb);
        /* QK-norm (qwen3.cpp:215-224) then RoPE NEOX */
        orc_rms_norm(q, L->q_norm, q, Tcur * c->n_head, HD, c->eps);
        orc_rms_norm(k, L->k_norm, k, Tcur * c->n_head_kv, HD, c->eps);
        for (int64_t t = 0; t < Tcur; ++t) {
            orc_rope_neox(q + t * Dq, q + t * Dq, c->n_head, HD, pos0 + (int32_t)t, c->freq_base);
            orc_rope_neox(k + t * Dkv, k + t * Dkv, c->n_head_kv, HD, pos0 + (int32_t)t, c->freq_base);
            /* set_rows fp32 -> fp16 at cell pos0+t (ops.cpp:135-181) */
            for (int64_t d = 0; d < Dkv; ++d) {
                L->kc[(int64_t)(pos0 + t) * Dkv + d] = orc_fp32_to_fp16(k[t * Dkv + d]);
                L->vc[(int64_t)(pos0 + t) * Dkv + d] = orc_fp32_to_fp16(v[t * Dkv + d]);
            }
        }
        orc_flash_attn_mt(q, L->kc, L->vc, kv_len, Tcur, c->n_head, c->n_head_kv, HD, 1.0f / sqrtf((float)HD),
                          fa_mode, att, m->n_threads);
        matmul_rows_cols_split(m, L->wo, att, o, Tcur, E, Dq, qb);
        if (l == c->n_layer - 1 && Tcur > 1) { /* keep the last row only (qwen3.cpp:235-238) */
            memmove(o, o + (Tcur - 1) * E, E * 4);
            memmove(x, x + (Tcur - 1) * E, E * 4);
            Tcur = 1;
        }
        for (int64_t i = 0; i < Tcur * E; ++i) x[i] = o[i] + x[i];
        orc_rms_norm(x, L->ffn_norm, h, Tcur, E, c->eps);
        matmul_rows(m, L->wgate, h, g, Tcur, c->n_ff, E, qb);
        matmul_rows(m, L->wup, h, u, Tcur, c->n_ff, E, qb);
        orc_swiglu(g, u, g, Tcur * c->n_ff);
        matmul_rows_cols_split(m, L->wdown, g, o, Tcur, E, c->n_ff, qb);
        for (int64_t i = 0; i < Tcur * E; ++i) x[i] = o[i] + x[i];
    }
    if (rc == 0) {
        const float * xl = x + (Tcur - 1) * E;
        orc_rms_norm(xl, m->output_norm, h, 1, E, c->eps);
        if (hidden) memcpy(hidden, h, E * 4);
        orc_quantize_row_q8_0(h, qb, E);
        if (m->exact) orc_gemv_q4_0_q8_0_exact(m->output, qb, logits, c->n_vocab, E, m->n_threads);
        else orc_mul_mat_generic(m->output, qb, logits, c->n_vocab, E, m->n_threads);
    }
    free(x); free(h); free(q); free(k); free(v); free(att); free(g); free(u); free(o); free(kv_len); free(qb);
    return rc;
}

int32_t orc_argmax(const float * x, int64_t n) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; ++i) if (x[i] > x[best]) best = i;
    return (int32_t)best;
}
