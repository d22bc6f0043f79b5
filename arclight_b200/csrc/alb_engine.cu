// Qwen3 Q4_0 decode/prefill engine: the B200 counterpart of the reference's
// llm_model + nnml_cgraph + llm_kv_cache + decoding_context for one sequence.
//
// One engine per GPU (one process or thread per GPU).  With tp_size > 1 the
// weights are sharded exactly as the reference's NUMA tensor parallelism
// (model.cpp:21-130): Q/K/V and gate/up by output rows (whole heads / 32-row
// units), O and down by input columns, norms replicated, KV cache by KV head
// (cgraph.cpp:962-973); the reference's GATHER (ops.cpp:1465-1511) becomes an
// NCCL sum all-reduce of the residual stream after O and after down.  The lm
// head is sharded by vocabulary rows and the greedy argmax is an all-reduce
// MAX over (value, index) keys.
//
// A decode step is one CUDA graph (captured once): every kernel is launched as
// a programmatic dependent of the previous one, reads the token and position
// from device memory and writes the next token back, so a greedy loop needs
// no host round trip.  Prefill runs the same ops over a ubatch of T tokens.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "alb_common.cuh"
#include "alb_internal.h"
#include "alb_nccl.h"
#include "alb_wait.h"

namespace alb {
void normal_table_host(std::vector<float> & t);
uint64_t tensor_seed(uint64_t model_seed, int layer, int kind);
void rope_table_host(std::vector<float> & t, int32_t max_pos, int32_t head_dim, float freq_base);
cudaError_t gen_q4(uint8_t * W, int64_t N_total, int64_t K, int64_t dst_row0, int64_t dst_row_stride, int64_t n_rows,
                   uint64_t seed, int64_t src_row0, int64_t K_full, int64_t c0, const float * table, cudaStream_t st);
cudaError_t gen_norm(float * w, int64_t n, uint64_t seed, const float * table, cudaStream_t st);
cudaError_t gen_f16(uint16_t * dst, int64_t cells, int64_t row, int64_t full_row, int64_t col0, uint64_t seed,
                    const float * table, cudaStream_t st);

enum Kind { T_TOK_EMBD = 0, T_OUTPUT = 1, T_OUTPUT_NORM = 2, T_ATTN_NORM = 3, T_WQ = 4, T_WK = 5, T_WV = 6, T_WO = 7,
            T_Q_NORM = 8, T_K_NORM = 9, T_FFN_NORM = 10, T_GATE = 11, T_UP = 12, T_DOWN = 13 };

__global__ void k_advance(int32_t * tok, int32_t * pos, const int32_t * next, int32_t * out, int32_t * step, int32_t cap) {
    alb_pdl_wait();
    const int32_t n = *next;
    const int32_t s = *step;
    if (s < cap) out[s] = n;
    *step = s + 1;
    *tok = n;
    *pos = *pos + 1;
}
// GATHER (ops.cpp:1465-1511, nnml_vec_add_f32 arm.cpp:2435-2451) then ADD of
// the residual (qwen3.cpp:241,270): x[i] = (((p_0 + p_1) + ...) + p_{n-1}) + x[i],
// the rank partials added in rank order in fp32, as the reference's nodes.
__global__ void k_gather_add(float * x, const float * parts, int n_parts, int64_t count) {
    alb_pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        float acc = parts[i];
        for (int j = 1; j < n_parts; ++j) acc = __fadd_rn(acc, parts[(int64_t)j * count + i]);
        x[i] = __fadd_rn(acc, x[i]);
    }
}
}  // namespace alb

using namespace alb;

struct alb_engine {
    alb_qwen3_config c;
    uint64_t seed = 0;
    int32_t max_ctx = 0, max_ub = 0, rank = 0, tp = 1;
    int E = 0, Hq = 0, Hkv = 0, F = 0, V = 0, Dq = 0, Dkv = 0, Nqkv = 0, v0 = 0;
    int dev = 0;
    cudaStream_t st = nullptr;
    void * comm = nullptr;
    bool comm_failed = false;        // the communicator was aborted: no further steps
    double comm_timeout_ms = 0.0;    // bounded wait for steps with collectives
    struct Layer {
        uint8_t * qkv = nullptr, * o = nullptr, * gu = nullptr, * down = nullptr;
        float * an = nullptr, * fn = nullptr, * qn = nullptr, * kn = nullptr;
        uint16_t * kc = nullptr, * vc = nullptr;
    };
    std::vector<Layer> layers;
    uint8_t * tok = nullptr, * out_w = nullptr;
    const uint8_t * lm_W = nullptr;                 // lm head rows of this rank (a view of the token table when tied)
    float * out_norm = nullptr, * table = nullptr, * rope = nullptr;
    float * x = nullptr, * qkv = nullptr, * q = nullptr, * att = nullptr, * h = nullptr, * logits = nullptr;
    float * part = nullptr, * part_all = nullptr;   // TP: this rank's O / down partial, all ranks' partials
    float * xn = nullptr;                           // prefill: RMS-normalized rows
    void * xq = nullptr;                            // decode: block_q8_0 input of the next mat-vec
    void * pg_ws = nullptr;                         // prefill: quantized activations of the mat-mul
    float * fa_sws = nullptr;                       // prefill: the attention's score workspace
    int32_t * tok_dev = nullptr, * pos_dev = nullptr, * next_dev = nullptr, * step_dev = nullptr, * gen_out = nullptr;
    int32_t gen_cap = 0;
    unsigned long long * key = nullptr;
    void * am_scratch = nullptr;
    float * fa_ws = nullptr;
    int fa_S_decode = 1;
    bool fa_cluster = false;    // decode attention: one cluster launch per layer (max_ctx small enough)
    size_t fa_ws_bytes = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t gexec = nullptr;
    bool graph_loop = false;        // graph also advances token/pos (greedy loop)
    std::vector<void *> allocs;
    size_t bytes = 0;
    int32_t * pinned = nullptr;     // host staging for the e2e path
    int launches_per_step = 0;

    template <typename T> int alloc(T ** p, size_t n) {
        void * v = nullptr;
        const size_t b = (n * sizeof(T) + 255) & ~(size_t)255;
        if (cudaMalloc(&v, b) != cudaSuccess) { alb_set_last_error_msg("cudaMalloc failed (engine)"); return ALB_ERR_OOM; }
        allocs.push_back(v);
        bytes += b;
        *p = static_cast<T *>(v);
        return ALB_OK;
    }
};

#define ALB_TRY(expr) do { int r__ = (expr); if (r__ != ALB_OK) return r__; } while (0)

// TP: the reference's GATHER of the rank partials (e->part) then the residual
// ADD, as an all-gather plus an ordered sum (same fp32 additions in the same
// order on every rank, for any number of ranks).
static int engine_gather_add_x(alb_engine * e, int64_t T, bool pdl) {
    const size_t n = (size_t)T * e->E;
    ALB_TRY(nccl_allgather_f32(e->comm, e->part, e->part_all, n, e->st));
    const int blocks = (int)((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024);
    ALB_CUDA_TRY(alb_launch(k_gather_add, dim3(blocks), dim3(256), 0, e->st, pdl, e->x, (const float *)e->part_all,
                            e->tp, (int64_t)n));
    return ALB_OK;
}

// One ubatch of T tokens (token ids in tok_dev[0..T), first position in pos_dev)
// through the whole model, ending with the greedy next token in next_dev.
static int engine_forward(alb_engine * e, int64_t T, bool pdl, int ncap_prefill = 0) {
    const alb_qwen3_config & c = e->c;
    cudaStream_t st = e->st;
    int launches = 0;
    ALB_CUDA_TRY(launch_embed(e->tok, c.n_vocab, e->E, e->tok_dev, (int)T, e->x, e->key, pdl, st));
    ++launches;
    auto gemv = [&](const uint8_t * W, int64_t N, int64_t K, int in, const void * x, const float * nw, int out,
                    float * y, const float * res) -> cudaError_t {
        GemvArgs a;
        a.W = W; a.N = N; a.K = K;
        a.in_mode = in; a.x = x; a.norm_w = nw; a.eps = c.eps;
        a.out_mode = out; a.y = y; a.residual = res; a.pdl = pdl;
        ++launches;
        // decode: records already in x (attention merge, gate/up epilogue), or
        // RMSNorm + quantization in the mat-vec's prologue, which overlaps the
        // weight stages the producer warp has in flight
        if (T == 1) return launch_gemv(a, st);
        // prefill: RMSNorm rows (when asked), then the tensor-core mat-mul
        const float * xin = static_cast<const float *>(x);
        if (in == GEMV_IN_F32_RMS) {
            const cudaError_t re = launch_rms_norm(xin, nw, e->xn, T, K, c.eps, pdl, st);
            if (re != cudaSuccess) return re;
            xin = e->xn;
            ++launches;
        }
        ++launches;   // activation quantizer
        return launch_prefill_gemm(W, N, K, xin, nullptr, T, y, out == GEMV_OUT_SWIGLU ? N / 2 : N, res,
                                   out == GEMV_OUT_SWIGLU, e->pg_ws, device_error_ptr(), pdl, st);
    };
    const int S = T == 1 ? e->fa_S_decode : 1;
    for (int l = 0; l < c.n_layer; ++l) {
        alb_engine::Layer & L = e->layers[l];
        ALB_CUDA_TRY(gemv(L.qkv, e->Nqkv, e->E, GEMV_IN_F32_RMS, e->x, L.an, GEMV_OUT_PLAIN, e->qkv, nullptr));
        QkvArgs qa;
        qa.qkv = e->qkv; qa.qkv_stride = e->Nqkv; qa.Hq = e->Hq; qa.Hkv = e->Hkv; qa.T = (int)T;
        qa.q_norm = L.qn; qa.k_norm = L.kn; qa.eps = c.eps; qa.rope = reinterpret_cast<const float2 *>(e->rope);
        qa.pos_dev = e->pos_dev; qa.q_out = e->q; qa.kc = L.kc; qa.vc = L.vc; qa.pdl = pdl;
        FlashArgs fa;
        fa.q = e->q; fa.kc = L.kc; fa.vc = L.vc; fa.Hq = e->Hq; fa.Hkv = e->Hkv; fa.T = (int)T;
        fa.pos_dev = e->pos_dev; fa.scale = 1.0f / sqrtf((float)c.head_dim); fa.S = S; fa.ws = e->fa_ws;
        fa.ncap = T == 1 ? e->max_ctx : ncap_prefill;
        fa.out = e->att; fa.pdl = pdl;
        if (T == 1) {
            // decode: QK-norm + RoPE + K/V store inside the split score kernel; the
            // last CTA of each KV head writes the O projection's Q8_0 input records
            fa.xq = e->xq;
            ALB_CUDA_TRY(launch_attn_decode(fa, qa, e->fa_cluster, st));
            launches += e->fa_cluster ? 1 : 2;   // the cluster kernel, or scores + P.V
        } else {
            ALB_CUDA_TRY(launch_qk_norm_rope_kv(qa, st));
            fa.sws = e->fa_sws;   // sized for max_ubatch tokens over max_ctx cells (ncap <= max_ctx)
            ALB_CUDA_TRY(launch_flash_attn(fa, st));
            launches += 2;   // QK-norm/RoPE + the prefill attention
        }
        const int o_in = T == 1 ? GEMV_IN_Q8 : GEMV_IN_F32;
        const void * o_x = T == 1 ? e->xq : static_cast<const void *>(e->att);
        if (e->tp == 1) {
            ALB_CUDA_TRY(gemv(L.o, e->E, e->Dq, o_in, o_x, nullptr, GEMV_OUT_PLAIN, e->x, e->x));
        } else {
            ALB_CUDA_TRY(gemv(L.o, e->E, e->Dq, o_in, o_x, nullptr, GEMV_OUT_PLAIN, e->part, nullptr));
            ALB_TRY(engine_gather_add_x(e, T, pdl));
        }
        ALB_CUDA_TRY(gemv(L.gu, 2 * (int64_t)e->F, e->E, GEMV_IN_F32_RMS, e->x, L.fn, GEMV_OUT_SWIGLU, e->h, nullptr));
        // down: the SwiGLU output quantized in the mat-vec's prologue (decode)
        // or by the mat-mul's quantizer (prefill)
        if (e->tp == 1) {
            ALB_CUDA_TRY(gemv(L.down, e->E, e->F, GEMV_IN_F32, e->h, nullptr, GEMV_OUT_PLAIN, e->x, e->x));
        } else {
            ALB_CUDA_TRY(gemv(L.down, e->E, e->F, GEMV_IN_F32, e->h, nullptr, GEMV_OUT_PLAIN, e->part, nullptr));
            ALB_TRY(engine_gather_add_x(e, T, pdl));
            launches += 2;   // the two k_gather_add (the NCCL all-gathers are NCCL's kernels)
        }
    }
    // final norm + lm_head on the last token (qwen3.cpp:235-238, 266-274) through
    // the generic mul_mat's vec_dot chains (the output matrix is not repacked,
    // model.cpp:342-353), with the greedy argmax (sampler.cpp:34-36) fused: every
    // CTA max-reduces its (logit, index) keys into e->key (cleared by the
    // embedding kernel of this pass); on one GPU the last CTA writes the token
    {
        GemvArgs a;
        a.W = e->lm_W; a.N = e->V; a.K = e->E;
        a.in_mode = GEMV_IN_F32_RMS; a.x = e->x + (size_t)(T - 1) * e->E; a.norm_w = e->out_norm; a.eps = c.eps;
        a.out_mode = GEMV_OUT_LOGITS; a.y = e->logits; a.pdl = pdl;
        a.ctas = 2 * alb_sm_count();   // the step's last mat-vec: both halves of every SM
        a.key = e->key; a.idx_base = e->v0;
        a.ticket = reinterpret_cast<int *>(e->am_scratch);
        a.next = e->tp == 1 ? e->next_dev : nullptr;
        ALB_CUDA_TRY(launch_gemv(a, st));
        ++launches;
    }
    if (e->tp > 1) {
        // the shards' keys: all-reduce MAX, then the index (first maximum overall)
        ALB_TRY(nccl_allreduce(e->comm, e->key, e->key, 1, 1, 1, st));
        ALB_CUDA_TRY(launch_key_to_index(e->key, e->next_dev, false, st));
        launches += 1;   // key_to_index (the all-reduce is NCCL's)
    }
    e->launches_per_step = launches;
    return ALB_OK;
}

static int engine_build_graph(alb_engine * e) {
    if (e->gexec) return ALB_OK;
    ALB_CUDA_TRY(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
    int rc = engine_forward(e, 1, true);
    if (rc == ALB_OK) {
        const cudaError_t le = alb_launch(k_advance, dim3(1), dim3(1), 0, e->st, true, e->tok_dev, e->pos_dev,
                                          (const int32_t *)e->next_dev, e->gen_out, e->step_dev, e->gen_cap);
        if (le != cudaSuccess) { alb_set_last_cuda_error(le, "k_advance"); rc = ALB_ERR_CUDA; }
    }
    cudaGraph_t g = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(e->st, &g);
    if (rc != ALB_OK) { if (g) cudaGraphDestroy(g); return rc; }
    ALB_CUDA_TRY(ce);
    e->graph = g;
    ALB_CUDA_TRY(cudaGraphInstantiate(&e->gexec, g, 0));
    e->launches_per_step += 1;
    return ALB_OK;
}

static int engine_init_weights(alb_engine * e) {
    const alb_qwen3_config & c = e->c;
    cudaStream_t st = e->st;
    std::vector<float> tab;
    normal_table_host(tab);
    ALB_TRY(e->alloc(&e->table, tab.size()));
    ALB_CUDA_TRY(cudaMemcpyAsync(e->table, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice, st));
    const int64_t E = e->E, HD = c.head_dim;
    const int64_t Dq_full = (int64_t)c.n_head * HD, Dkv_full = (int64_t)c.n_head_kv * HD;
    auto seed = [&](int layer, int kind) { return tensor_seed(e->seed, layer, kind); };
    // token table: full on every rank (embedding lookup; tied lm_head shard is a view)
    ALB_TRY(e->alloc(&e->tok, q4_gpu_bytes(c.n_vocab, E)));
    ALB_CUDA_TRY(gen_q4(e->tok, c.n_vocab, E, 0, 1, c.n_vocab, seed(-1, T_TOK_EMBD), 0, E, 0, e->table, st));
    if (c.tied) {
        e->lm_W = e->tok + (size_t)e->v0 * q4_row_bytes(E);   // this rank's vocabulary rows
    } else {
        ALB_TRY(e->alloc(&e->out_w, q4_gpu_bytes(e->V, E)));
        ALB_CUDA_TRY(gen_q4(e->out_w, e->V, E, 0, 1, e->V, seed(-1, T_OUTPUT), e->v0, E, 0, e->table, st));
        e->lm_W = e->out_w;
    }
    ALB_TRY(e->alloc(&e->out_norm, E));
    ALB_CUDA_TRY(gen_norm(e->out_norm, E, seed(-1, T_OUTPUT_NORM), e->table, st));
    e->layers.resize(c.n_layer);
    const int64_t cells = e->max_ctx;
    // one buffer for every layer's mat-vec weights, in the decode step's order
    // (QKV, O, gate/up, down of each layer: one sequential stream per token)
    auto a256 = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t b_qkv = a256(q4_gpu_bytes(e->Nqkv, E)), b_o = a256(q4_gpu_bytes(E, e->Dq));
    const size_t b_gu = a256(q4_gpu_bytes(2 * (int64_t)e->F, E)), b_down = a256(q4_gpu_bytes(E, e->F));
    const size_t b_layer = b_qkv + b_o + b_gu + b_down;
    uint8_t * arena = nullptr;
    ALB_TRY(e->alloc(&arena, b_layer * (size_t)c.n_layer));
    for (int l = 0; l < c.n_layer; ++l) {
        alb_engine::Layer & L = e->layers[l];
        L.qkv = arena + (size_t)l * b_layer;
        L.o = L.qkv + b_qkv;
        L.gu = L.o + b_o;
        L.down = L.gu + b_gu;
        ALB_CUDA_TRY(gen_q4(L.qkv, e->Nqkv, E, 0, 1, e->Dq, seed(l, T_WQ), (int64_t)e->rank * e->Dq, E, 0, e->table, st));
        ALB_CUDA_TRY(gen_q4(L.qkv, e->Nqkv, E, e->Dq, 1, e->Dkv, seed(l, T_WK), (int64_t)e->rank * e->Dkv, E, 0, e->table, st));
        ALB_CUDA_TRY(gen_q4(L.qkv, e->Nqkv, E, e->Dq + e->Dkv, 1, e->Dkv, seed(l, T_WV), (int64_t)e->rank * e->Dkv, E, 0,
                            e->table, st));
        ALB_CUDA_TRY(gen_q4(L.o, E, e->Dq, 0, 1, E, seed(l, T_WO), 0, Dq_full, (int64_t)e->rank * e->Dq, e->table, st));
        ALB_CUDA_TRY(gen_q4(L.gu, 2 * (int64_t)e->F, E, 0, 2, e->F, seed(l, T_GATE), (int64_t)e->rank * e->F, E, 0, e->table, st));
        ALB_CUDA_TRY(gen_q4(L.gu, 2 * (int64_t)e->F, E, 1, 2, e->F, seed(l, T_UP), (int64_t)e->rank * e->F, E, 0, e->table, st));
        ALB_CUDA_TRY(gen_q4(L.down, E, e->F, 0, 1, E, seed(l, T_DOWN), 0, c.n_ff, (int64_t)e->rank * e->F, e->table, st));
        ALB_TRY(e->alloc(&L.an, E));
        ALB_TRY(e->alloc(&L.fn, E));
        ALB_TRY(e->alloc(&L.qn, HD));
        ALB_TRY(e->alloc(&L.kn, HD));
        ALB_CUDA_TRY(gen_norm(L.an, E, seed(l, T_ATTN_NORM), e->table, st));
        ALB_CUDA_TRY(gen_norm(L.fn, E, seed(l, T_FFN_NORM), e->table, st));
        ALB_CUDA_TRY(gen_norm(L.qn, HD, seed(l, T_Q_NORM), e->table, st));
        ALB_CUDA_TRY(gen_norm(L.kn, HD, seed(l, T_K_NORM), e->table, st));
        ALB_TRY(e->alloc(&L.kc, (size_t)cells * e->Dkv));
        ALB_TRY(e->alloc(&L.vc, (size_t)cells * e->Dkv));
        ALB_CUDA_TRY(cudaMemsetAsync(L.kc, 0, (size_t)cells * e->Dkv * 2, st));
        ALB_CUDA_TRY(cudaMemsetAsync(L.vc, 0, (size_t)cells * e->Dkv * 2, st));
        (void)Dkv_full;
    }
    std::vector<float> rt;
    rope_table_host(rt, e->max_ctx, (int)HD, c.freq_base);
    ALB_TRY(e->alloc(&e->rope, rt.size()));
    ALB_CUDA_TRY(cudaMemcpyAsync(e->rope, rt.data(), rt.size() * 4, cudaMemcpyHostToDevice, st));
    ALB_CUDA_TRY(cudaStreamSynchronize(st));
    return ALB_OK;
}

static int engine_init_acts(alb_engine * e) {
    const int64_t U = e->max_ub;
    ALB_TRY(e->alloc(&e->x, U * e->E));
    ALB_TRY(e->alloc(&e->qkv, U * e->Nqkv));
    ALB_TRY(e->alloc(&e->q, U * e->Dq));
    ALB_TRY(e->alloc(&e->att, U * e->Dq));
    ALB_TRY(e->alloc(&e->h, U * e->F));
    {
        int64_t kmax = e->E > e->Dq ? e->E : e->Dq;
        if (e->F > kmax) kmax = e->F;
        uint8_t * q8 = nullptr;
        ALB_TRY(e->alloc(&q8, (size_t)(kmax / 32) * 34));
        e->xq = q8;
    }
    if (U > 1) {
        ALB_TRY(e->alloc(&e->xn, U * e->E));
        int64_t kmax = e->E > e->Dq ? e->E : e->Dq;
        if (e->F > kmax) kmax = e->F;
        uint8_t * w = nullptr;
        ALB_TRY(e->alloc(&w, prefill_ws_bytes(U, kmax)));
        e->pg_ws = w;
        // prefill attention scores, written by pass 1 and read by pass 2
        uint8_t * sw = nullptr;
        ALB_TRY(e->alloc(&sw, fa_prefill_scores_bytes(e->Hq, e->Hkv, (int)U, e->max_ctx)));
        e->fa_sws = reinterpret_cast<float *>(sw);
    }
    if (e->tp > 1) {
        ALB_TRY(e->alloc(&e->part, U * e->E));
        ALB_TRY(e->alloc(&e->part_all, (int64_t)e->tp * U * e->E));
    }
    ALB_TRY(e->alloc(&e->logits, (size_t)e->V));
    ALB_TRY(e->alloc(&e->tok_dev, (size_t)U));
    ALB_TRY(e->alloc(&e->pos_dev, 1));
    ALB_TRY(e->alloc(&e->next_dev, 1));
    ALB_TRY(e->alloc(&e->step_dev, 1));
    e->gen_cap = 1 << 16;
    ALB_TRY(e->alloc(&e->gen_out, (size_t)e->gen_cap));
    ALB_TRY(e->alloc(&e->key, 1));
    uint8_t * scr = nullptr;
    ALB_TRY(e->alloc(&scr, 1024));
    e->am_scratch = scr;
    // decode split-K: 4 CTAs per SM (the split kernels' staging ring allows four) over the local KV heads
    int S = (4 * alb_sm_count() + e->Hkv - 1) / e->Hkv;
    if (S > 1024) S = 1024;
    e->fa_S_decode = S;
    e->fa_cluster = e->max_ctx <= attn_decode_cluster_max_cells();
    e->fa_ws_bytes = flash_attn_ws_bytes(e->Hq, e->Hkv, 1, S, e->max_ctx);   // prefill ubatches need none
    uint8_t * ws = nullptr;
    ALB_TRY(e->alloc(&ws, e->fa_ws_bytes));
    e->fa_ws = reinterpret_cast<float *>(ws);
    ALB_CUDA_TRY(cudaMemsetAsync(ws, 0, e->fa_ws_bytes, e->st));
    ALB_CUDA_TRY(cudaMemsetAsync(scr, 0, 1024, e->st));
    ALB_CUDA_TRY(cudaMemsetAsync(e->step_dev, 0, 4, e->st));
    ALB_CUDA_TRY(cudaMallocHost(&e->pinned, 64));
    ALB_CUDA_TRY(cudaStreamSynchronize(e->st));
    return ALB_OK;
}

static void engine_free(alb_engine * e) {
    if (!e) return;
    cudaSetDevice(e->dev);
    if (e->st) cudaStreamSynchronize(e->st);
    if (e->gexec) cudaGraphExecDestroy(e->gexec);
    if (e->graph) cudaGraphDestroy(e->graph);
    for (void * p : e->allocs) cudaFree(p);
    if (e->pinned) cudaFreeHost(e->pinned);
    if (e->comm) nccl_destroy(e->comm, false);
    if (e->st) cudaStreamDestroy(e->st);
    delete e;
}

extern "C" int alb_nccl_unique_id(void * out128) {
    ALB_CHECK_ARG(out128);
    return nccl_unique_id(out128);
}

// Communicator of the tensor-parallel clique for callers that run the op-level
// ABI themselves (the reference's GATHER, ops.cpp:1465-1511, becomes a sum
// all-reduce or an all-gather followed by an ordered sum).
struct alb_comm {
    void * nccl = nullptr;
    int dev = 0;
};

extern "C" int alb_comm_create(const void * nccl_id, int32_t rank, int32_t size, int32_t device, alb_comm ** out) {
    ALB_CHECK_ARG(nccl_id && out && size >= 1 && rank >= 0 && rank < size && device >= 0);
    *out = nullptr;
    ALB_CUDA_TRY(cudaSetDevice(device));
    alb_comm * c = new alb_comm();
    c->dev = device;
    const int rc = nccl_init(&c->nccl, rank, size, nccl_id);
    if (rc != ALB_OK) { delete c; return rc; }
    *out = c;
    return ALB_OK;
}

extern "C" int alb_comm_destroy(alb_comm * c) {
    if (!c) return ALB_OK;
    cudaSetDevice(c->dev);
    nccl_destroy(c->nccl, false);
    delete c;
    return ALB_OK;
}

extern "C" int alb_allreduce_sum_f32(alb_comm * c, const float * src, float * dst, int64_t n, void * stream) {
    ALB_CHECK_ARG(c && src && dst && n > 0);
    return nccl_allreduce(c->nccl, src, dst, (size_t)n, 0, 0, (cudaStream_t)stream);
}

extern "C" int alb_allgather_f32(alb_comm * c, const float * src, float * dst, int64_t n, void * stream) {
    ALB_CHECK_ARG(c && src && dst && n > 0);
    return nccl_allgather_f32(c->nccl, src, dst, (size_t)n, (cudaStream_t)stream);
}

extern "C" int alb_engine_create(const alb_qwen3_config * cfg, uint64_t seed, int32_t max_ctx, int32_t max_ubatch,
                                 int32_t tp_rank, int32_t tp_size, const void * nccl_id, int32_t device,
                                 alb_engine ** out) {
    ALB_CHECK_ARG(cfg && out && max_ctx > 0 && max_ubatch > 0 && tp_size >= 1 && tp_rank >= 0 && tp_rank < tp_size);
    ALB_CHECK_ARG(cfg->head_dim == 128 && cfg->n_layer > 0 && cfg->n_embd % 32 == 0 && cfg->n_embd <= 12288);
    ALB_CHECK_ARG(cfg->n_head % tp_size == 0 && cfg->n_head_kv % tp_size == 0 && cfg->n_head % cfg->n_head_kv == 0);
    ALB_CHECK_ARG(cfg->n_ff % (32 * tp_size) == 0 && cfg->n_vocab % tp_size == 0);
    ALB_CHECK_ARG(tp_size == 1 || nccl_id);
    *out = nullptr;
    const int rc0 = alb_device_check(device);
    if (rc0 != ALB_OK) return rc0;
    ALB_CUDA_TRY(cudaSetDevice(device));
    // The per-device error word is created by a synchronous allocation on first
    // use; that first use must not fall inside the decode-graph capture.
    if (!device_error_ptr()) { alb_set_last_error_msg("device error word: allocation failed"); return ALB_ERR_CUDA; }
    alb_engine * e = new alb_engine();
    e->c = *cfg; e->seed = seed; e->max_ctx = max_ctx; e->max_ub = max_ubatch;
    e->rank = tp_rank; e->tp = tp_size; e->dev = device;
    e->E = cfg->n_embd;
    e->Hq = cfg->n_head / tp_size; e->Hkv = cfg->n_head_kv / tp_size;
    e->F = cfg->n_ff / tp_size; e->V = cfg->n_vocab / tp_size; e->v0 = e->V * tp_rank;
    e->Dq = e->Hq * cfg->head_dim; e->Dkv = e->Hkv * cfg->head_dim;
    e->Nqkv = e->Dq + 2 * e->Dkv;
    int rc = ALB_OK;
    if (cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking) != cudaSuccess) rc = ALB_ERR_CUDA;
    if (rc == ALB_OK && tp_size > 1) rc = nccl_init(&e->comm, tp_rank, tp_size, nccl_id);
    if (const char * v = getenv("ALB_NCCL_TIMEOUT_MS")) e->comm_timeout_ms = atof(v);
    if (e->comm_timeout_ms <= 0.0) e->comm_timeout_ms = 120000.0;
    if (rc == ALB_OK) rc = engine_init_weights(e);
    if (rc == ALB_OK) rc = engine_init_acts(e);
    if (rc != ALB_OK) { engine_free(e); return rc; }
    *out = e;
    return ALB_OK;
}

extern "C" int alb_engine_destroy(alb_engine * e) {
    engine_free(e);
    return ALB_OK;
}

extern "C" size_t alb_engine_device_bytes(const alb_engine * e) { return e ? e->bytes : 0; }

extern "C" int alb_engine_reset(alb_engine * e) {
    ALB_CHECK_ARG(e);
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    for (auto & L : e->layers) {
        ALB_CUDA_TRY(cudaMemsetAsync(L.kc, 0, (size_t)e->max_ctx * e->Dkv * 2, e->st));
        ALB_CUDA_TRY(cudaMemsetAsync(L.vc, 0, (size_t)e->max_ctx * e->Dkv * 2, e->st));
    }
    ALB_CUDA_TRY(cudaStreamSynchronize(e->st));
    return ALB_OK;
}

// Wait for the engine's stream.  A tensor-parallel engine waits boundedly: a
// peer that stops answering within ALB_NCCL_TIMEOUT_MS (default 120 s), or an
// asynchronous NCCL error, aborts the communicator so the collective kernels
// spinning on that peer return; the engine then refuses further steps.
static int engine_sync(alb_engine * e) {
    if (!e->comm) {
        ALB_CUDA_TRY(cudaStreamSynchronize(e->st));
        return ALB_OK;
    }
    cudaError_t serr = cudaSuccess;
    auto query = [&]() {
        const cudaError_t q = cudaStreamQuery(e->st);
        if (q == cudaSuccess) return 0;
        if (q == cudaErrorNotReady) return 1;
        serr = q;
        return -1;
    };
    const WaitResult w = bounded_wait(query, [&]() { return nccl_async_error(e->comm) != ALB_OK ? 1 : 0; },
                                      e->comm_timeout_ms);
    (void)cudaGetLastError();   // the polls' not-ready answers
    if (w == WaitResult::kDone) return ALB_OK;
    if (w == WaitResult::kStreamError) {
        alb_set_last_cuda_error(serr, "engine stream");
        return ALB_ERR_CUDA;
    }
    nccl_destroy(e->comm, true);   // ncclCommAbort: the collectives in flight return
    e->comm = nullptr;
    e->comm_failed = true;
    bounded_wait(query, []() { return 0; }, e->comm_timeout_ms);
    (void)cudaGetLastError();
    alb_set_last_error_msg(w == WaitResult::kTimeout
                               ? "tensor-parallel peer did not answer within ALB_NCCL_TIMEOUT_MS: communicator aborted"
                               : "NCCL reported an error: communicator aborted");
    return w == WaitResult::kTimeout ? ALB_ERR_TIMEOUT : ALB_ERR_NCCL;
}

static int engine_usable(const alb_engine * e) {
    if (e->comm_failed) {
        alb_set_last_error_msg("the engine's communicator was aborted; destroy the engine");
        return ALB_ERR_NCCL;
    }
    return ALB_OK;
}

// decoding_context::decode / process_ubatch (context.cpp:74-205) for a prompt
// chunk: tokens at positions [pos0, pos0 + n), split into ubatches of max_ubatch.
extern "C" int alb_engine_prefill(alb_engine * e, const int32_t * tokens, int32_t n, int32_t pos0,
                                  int32_t * next_token) {
    ALB_CHECK_ARG(e && tokens && n > 0 && pos0 >= 0 && (int64_t)pos0 + n <= e->max_ctx);
    ALB_TRY(engine_usable(e));
    for (int32_t i = 0; i < n; ++i) ALB_CHECK_ARG(tokens[i] >= 0 && tokens[i] < e->c.n_vocab);
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    for (int32_t off = 0; off < n; off += e->max_ub) {
        const int32_t T = (n - off) < e->max_ub ? (n - off) : e->max_ub;
        const int32_t p = pos0 + off;
        ALB_CUDA_TRY(cudaMemcpyAsync(e->tok_dev, tokens + off, (size_t)T * 4, cudaMemcpyHostToDevice, e->st));
        ALB_CUDA_TRY(cudaMemcpyAsync(e->pos_dev, &p, 4, cudaMemcpyHostToDevice, e->st));
        ALB_TRY(engine_sync(e));   // pageable sources: keep them alive
        ALB_TRY(engine_forward(e, T, false, p + T));
    }
    ALB_CUDA_TRY(cudaMemcpyAsync(e->pinned, e->next_dev, 4, cudaMemcpyDeviceToHost, e->st));
    ALB_TRY(engine_sync(e));
    if (next_token) *next_token = e->pinned[0];
    return ALB_OK;
}

// One greedy decode step (context.cpp:51-67): token at position pos.  Host
// buffers in and out: 8 bytes H2D (token, pos), 4 bytes D2H (next token).
extern "C" int alb_engine_decode(alb_engine * e, int32_t token, int32_t pos, int32_t * next_token) {
    ALB_CHECK_ARG(e && token >= 0 && token < e->c.n_vocab && pos >= 0 && pos < e->max_ctx);
    ALB_TRY(engine_usable(e));
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    ALB_TRY(engine_build_graph(e));
    e->pinned[0] = token;
    e->pinned[1] = pos;
    ALB_CUDA_TRY(cudaMemcpyAsync(e->tok_dev, &e->pinned[0], 4, cudaMemcpyHostToDevice, e->st));
    ALB_CUDA_TRY(cudaMemcpyAsync(e->pos_dev, &e->pinned[1], 4, cudaMemcpyHostToDevice, e->st));
    ALB_CUDA_TRY(cudaGraphLaunch(e->gexec, e->st));
    ALB_CUDA_TRY(cudaMemcpyAsync(&e->pinned[2], e->next_dev, 4, cudaMemcpyDeviceToHost, e->st));
    ALB_TRY(engine_sync(e));
    if (next_token) *next_token = e->pinned[2];
    return ALB_OK;
}

// Device-resident greedy loop: n_steps graph replays starting from (token, pos);
// every step's next token is appended on the device.  If tokens_out is non-null
// the generated tokens are copied back at the end.  Stream ordered, no host
// round trip between steps.
extern "C" int alb_engine_decode_loop(alb_engine * e, int32_t token, int32_t pos, int32_t n_steps,
                                      int32_t * tokens_out, int32_t sync) {
    ALB_CHECK_ARG(e && token >= 0 && token < e->c.n_vocab && pos >= 0 && n_steps > 0 && n_steps <= e->gen_cap);
    ALB_CHECK_ARG((int64_t)pos + n_steps <= e->max_ctx);
    ALB_TRY(engine_usable(e));
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    ALB_TRY(engine_build_graph(e));
    e->pinned[0] = token;
    e->pinned[1] = pos;
    e->pinned[2] = 0;
    ALB_CUDA_TRY(cudaMemcpyAsync(e->tok_dev, &e->pinned[0], 4, cudaMemcpyHostToDevice, e->st));
    ALB_CUDA_TRY(cudaMemcpyAsync(e->pos_dev, &e->pinned[1], 4, cudaMemcpyHostToDevice, e->st));
    ALB_CUDA_TRY(cudaMemcpyAsync(e->step_dev, &e->pinned[2], 4, cudaMemcpyHostToDevice, e->st));
    for (int32_t i = 0; i < n_steps; ++i) ALB_CUDA_TRY(cudaGraphLaunch(e->gexec, e->st));
    if (tokens_out) {
        ALB_CUDA_TRY(cudaMemcpyAsync(tokens_out, e->gen_out, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, e->st));
    }
    if (sync || tokens_out) ALB_TRY(engine_sync(e));
    return ALB_OK;
}

extern "C" int alb_engine_logits(alb_engine * e, float * host, int64_t n) {
    ALB_CHECK_ARG(e && host && n == e->V);
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    ALB_CUDA_TRY(cudaMemcpyAsync(host, e->logits, (size_t)n * 4, cudaMemcpyDeviceToHost, e->st));
    ALB_CUDA_TRY(cudaStreamSynchronize(e->st));
    return ALB_OK;
}

// The residual stream of the last forward pass (rows of its ubatch), for checks.
extern "C" int alb_engine_hidden(alb_engine * e, float * host, int64_t rows) {
    ALB_CHECK_ARG(e && host && rows > 0 && rows <= e->max_ub);
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    ALB_CUDA_TRY(cudaMemcpyAsync(host, e->x, (size_t)rows * e->E * 4, cudaMemcpyDeviceToHost, e->st));
    ALB_CUDA_TRY(cudaStreamSynchronize(e->st));
    return ALB_OK;
}

extern "C" int alb_engine_info(const alb_engine * e, int64_t * info, int32_t n) {
    ALB_CHECK_ARG(e && info && n >= 8);
    info[0] = e->V; info[1] = e->v0; info[2] = e->Hq; info[3] = e->Hkv; info[4] = e->F;
    info[5] = e->launches_per_step; info[6] = (int64_t)e->bytes; info[7] = e->fa_S_decode;
    return ALB_OK;
}

extern "C" void * alb_engine_stream(alb_engine * e) { return e ? (void *)e->st : nullptr; }

// Weight shard of (layer, kind) back in the reference's block_q4_0 layout
// [rows][K/32] (host buffer of rows*(K/32)*18 bytes) for parity checks of the
// generator; rows/cols describe this rank's shard.
extern "C" int alb_engine_weight_blocks(alb_engine * e, int32_t layer, int32_t kind, void * host, int64_t * rows,
                                        int64_t * cols) {
    ALB_CHECK_ARG(e && rows && cols && layer >= -1 && layer < e->c.n_layer);
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    const uint8_t * W = nullptr;
    int64_t N = 0, K = 0, r0 = 0, nr = 0, stride = 1;
    if (layer < 0) {
        if (kind == T_TOK_EMBD) { W = e->tok; N = e->c.n_vocab; K = e->E; nr = N; }
        else if (kind == T_OUTPUT && !e->c.tied) { W = e->out_w; N = e->V; K = e->E; nr = N; }
        else return ALB_ERR_INVALID;
    } else {
        alb_engine::Layer & L = e->layers[layer];
        switch (kind) {
            case T_WQ: W = L.qkv; N = e->Nqkv; K = e->E; r0 = 0; nr = e->Dq; break;
            case T_WK: W = L.qkv; N = e->Nqkv; K = e->E; r0 = e->Dq; nr = e->Dkv; break;
            case T_WV: W = L.qkv; N = e->Nqkv; K = e->E; r0 = e->Dq + e->Dkv; nr = e->Dkv; break;
            case T_WO: W = L.o; N = e->E; K = e->Dq; nr = N; break;
            case T_GATE: W = L.gu; N = 2 * (int64_t)e->F; K = e->E; r0 = 0; nr = e->F; stride = 2; break;
            case T_UP: W = L.gu; N = 2 * (int64_t)e->F; K = e->E; r0 = 1; nr = e->F; stride = 2; break;
            case T_DOWN: W = L.down; N = e->E; K = e->F; nr = N; break;
            default: return ALB_ERR_INVALID;
        }
    }
    *rows = nr; *cols = K;
    if (!host) return ALB_OK;
    uint8_t * tmp = nullptr;
    ALB_CUDA_TRY(cudaMalloc(&tmp, (size_t)N * (K / 32) * 18));
    int rc = alb_unpack_q4_0(tmp, W, N, K, e->st);
    if (rc == ALB_OK) {
        std::vector<uint8_t> all((size_t)N * (K / 32) * 18);
        if (cudaMemcpyAsync(all.data(), tmp, all.size(), cudaMemcpyDeviceToHost, e->st) != cudaSuccess ||
            cudaStreamSynchronize(e->st) != cudaSuccess) rc = ALB_ERR_CUDA;
        const size_t rb = (size_t)(K / 32) * 18;
        for (int64_t i = 0; rc == ALB_OK && i < nr; ++i)
            memcpy(static_cast<uint8_t *>(host) + i * rb, all.data() + (size_t)(r0 + i * stride) * rb, rb);
    }
    cudaFree(tmp);
    return rc;
}

extern "C" int alb_engine_norm_weights(alb_engine * e, int32_t layer, int32_t kind, float * host, int64_t n) {
    ALB_CHECK_ARG(e && host && layer >= -1 && layer < e->c.n_layer);
    const float * src = nullptr;
    int64_t len = 0;
    if (layer < 0 && kind == T_OUTPUT_NORM) { src = e->out_norm; len = e->E; }
    else if (layer >= 0) {
        alb_engine::Layer & L = e->layers[layer];
        if (kind == T_ATTN_NORM) { src = L.an; len = e->E; }
        if (kind == T_FFN_NORM) { src = L.fn; len = e->E; }
        if (kind == T_Q_NORM) { src = L.qn; len = 128; }
        if (kind == T_K_NORM) { src = L.kn; len = 128; }
    }
    ALB_CHECK_ARG(src && n == len);
    ALB_CUDA_TRY(cudaMemcpy(host, src, (size_t)n * 4, cudaMemcpyDeviceToHost));
    return ALB_OK;
}

// External weights (a model loaded from GGUF, model.cpp:355-474).  `host` holds
// the FULL tensor of (layer, kind) -- every rank's part -- in the reference
// block_q4_0 layout, [rows][cols / 32] blocks of 18 bytes; this rank keeps its
// shard the way slice_tensor (model.cpp:40-110) splits tensor-parallel weights:
// Q, K, V, gate, up and the untied lm head by rows, O and down by columns, the
// token table whole.  The shard is repacked on the device into the GPU layout
// in place of the generated weights (the captured step graph reads the same
// buffers, so nothing else changes).
extern "C" int alb_engine_set_weight_blocks(alb_engine * e, int32_t layer, int32_t kind, const void * host,
                                            int64_t rows, int64_t cols) {
    ALB_CHECK_ARG(e && host && rows > 0 && cols > 0 && cols % 32 == 0 && layer >= -1 && layer < e->c.n_layer);
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    uint8_t * W = nullptr;
    int64_t K = 0, r0 = 0, nr = 0, stride = 1;            // GPU buffer: columns, first row, shard rows, row step
    int64_t full_rows = 0, full_cols = 0, src_r0 = 0, src_c0 = 0;
    const int64_t tp = e->tp, rk = e->rank;
    if (layer < 0) {
        if (kind == T_TOK_EMBD) {
            W = e->tok; K = e->E; nr = e->c.n_vocab; full_rows = nr; full_cols = K;
        } else if (kind == T_OUTPUT && !e->c.tied) {
            W = e->out_w; K = e->E; nr = e->V; full_rows = (int64_t)e->V * tp; full_cols = K; src_r0 = e->v0;
        } else {
            return ALB_ERR_INVALID;
        }
    } else {
        alb_engine::Layer & L = e->layers[layer];
        switch (kind) {
            case T_WQ: W = L.qkv; K = e->E; r0 = 0; nr = e->Dq; break;
            case T_WK: W = L.qkv; K = e->E; r0 = e->Dq; nr = e->Dkv; break;
            case T_WV: W = L.qkv; K = e->E; r0 = e->Dq + e->Dkv; nr = e->Dkv; break;
            case T_GATE: W = L.gu; K = e->E; r0 = 0; nr = e->F; stride = 2; break;
            case T_UP: W = L.gu; K = e->E; r0 = 1; nr = e->F; stride = 2; break;
            case T_WO: W = L.o; K = e->Dq; nr = e->E; break;
            case T_DOWN: W = L.down; K = e->F; nr = e->E; break;
            default: return ALB_ERR_INVALID;
        }
        if (kind == T_WO || kind == T_DOWN) {   // column shards
            full_rows = nr; full_cols = K * tp; src_c0 = rk * K;
        } else {                                  // row shards
            full_rows = nr * tp; full_cols = K; src_r0 = rk * nr;
        }
    }
    ALB_CHECK_ARG(rows == full_rows && cols == full_cols);
    const size_t blk = 18, srb = (size_t)(full_cols / 32) * blk, drb = (size_t)(K / 32) * blk;
    std::vector<uint8_t> shard((size_t)nr * drb);
    for (int64_t i = 0; i < nr; ++i)
        memcpy(shard.data() + (size_t)i * drb, static_cast<const uint8_t *>(host) + (size_t)(src_r0 + i) * srb +
                                                    (size_t)(src_c0 / 32) * blk, drb);
    uint8_t * raw = nullptr, * gpu = nullptr;
    const size_t rowb = q4_row_bytes(K);
    int rc = ALB_OK;
    if (cudaMalloc(&raw, shard.size()) != cudaSuccess || cudaMalloc(&gpu, (size_t)nr * rowb) != cudaSuccess) rc = ALB_ERR_CUDA;
    if (rc == ALB_OK && cudaMemcpyAsync(raw, shard.data(), shard.size(), cudaMemcpyHostToDevice, e->st) != cudaSuccess)
        rc = ALB_ERR_CUDA;
    if (rc == ALB_OK) rc = alb_repack_q4_0(gpu, raw, nr, K, e->st);
    if (rc == ALB_OK && cudaMemcpy2DAsync(W + (size_t)r0 * rowb, (size_t)stride * rowb, gpu, rowb, rowb, (size_t)nr,
                                          cudaMemcpyDeviceToDevice, e->st) != cudaSuccess)
        rc = ALB_ERR_CUDA;
    if (rc == ALB_OK && cudaStreamSynchronize(e->st) != cudaSuccess) rc = ALB_ERR_CUDA;
    if (raw) cudaFree(raw);
    if (gpu) cudaFree(gpu);
    if (rc == ALB_ERR_CUDA) alb_set_last_error_msg(cudaGetErrorString(cudaGetLastError()));
    return rc;
}

// fp32 norm weights of (layer, kind) (every rank holds them whole).
extern "C" int alb_engine_set_norm_weights(alb_engine * e, int32_t layer, int32_t kind, const float * host, int64_t n) {
    ALB_CHECK_ARG(e && host && layer >= -1 && layer < e->c.n_layer);
    float * dst = nullptr;
    int64_t len = 0;
    if (layer < 0 && kind == T_OUTPUT_NORM) { dst = e->out_norm; len = e->E; }
    else if (layer >= 0) {
        alb_engine::Layer & L = e->layers[layer];
        if (kind == T_ATTN_NORM) { dst = L.an; len = e->E; }
        if (kind == T_FFN_NORM) { dst = L.fn; len = e->E; }
        if (kind == T_Q_NORM) { dst = L.qn; len = 128; }
        if (kind == T_K_NORM) { dst = L.kn; len = 128; }
    }
    ALB_CHECK_ARG(dst && n == len);
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    ALB_CUDA_TRY(cudaMemcpy(dst, host, (size_t)n * 4, cudaMemcpyHostToDevice));
    return ALB_OK;
}

// Times the decode step's Q4_0 mat-vec launches alone (all layers + lm head, in
// step order, PDL chained) from a CUDA graph replayed `reps` times.  Reports
// the mean duration per launch and the mean algorithmic bytes per launch
// (weights 18 B / 32 values + fp32 input + fp32 output).
// Times the prefill mat-muls of one ubatch of T = max_ubatch tokens alone (every
// layer's QKV, O, gate/up, down on the tensor cores, each with its activation
// quantizer), replayed `reps` times from a CUDA graph; reports the mean time per
// mat-mul launch and its int8 operations (2 * T * N * K).
extern "C" int alb_engine_time_prefill_gemm(alb_engine * e, int32_t reps, float * us_per_launch, double * ops_per_launch) {
    ALB_CHECK_ARG(e && reps > 0 && us_per_launch && ops_per_launch && e->max_ub > 1 && e->pg_ws);
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    const int64_t T = e->max_ub;
    struct G { const uint8_t * W; int64_t N, K; const float * x; float * y; bool swiglu; };
    std::vector<G> list;
    double ops = 0.0;
    for (int l = 0; l < e->c.n_layer; ++l) {
        alb_engine::Layer & L = e->layers[l];
        list.push_back({L.qkv, e->Nqkv, e->E, e->xn, e->qkv, false});
        list.push_back({L.o, e->E, e->Dq, e->att, e->qkv, false});
        list.push_back({L.gu, 2 * (int64_t)e->F, e->E, e->xn, e->h, true});
        list.push_back({L.down, e->E, e->F, e->h, e->qkv, false});
    }
    for (const G & g : list) ops += 2.0 * (double)T * (double)g.N * (double)g.K;
    ALB_CUDA_TRY(cudaMemsetAsync(e->xn, 0, (size_t)T * e->E * 4, e->st));
    ALB_CUDA_TRY(cudaMemsetAsync(e->att, 0, (size_t)T * e->Dq * 4, e->st));
    ALB_CUDA_TRY(cudaMemsetAsync(e->h, 0, (size_t)T * e->F * 4, e->st));
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    ALB_CUDA_TRY(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
    cudaError_t le = cudaSuccess;
    for (const G & a : list)
        if (le == cudaSuccess)
            le = launch_prefill_gemm(a.W, a.N, a.K, a.x, nullptr, T, a.y, a.swiglu ? a.N / 2 : a.N, nullptr, a.swiglu,
                                     e->pg_ws, device_error_ptr(), true, e->st);
    const cudaError_t ce = cudaStreamEndCapture(e->st, &g);
    ALB_CUDA_TRY(le);
    ALB_CUDA_TRY(ce);
    ALB_CUDA_TRY(cudaGraphInstantiate(&ge, g, 0));
    cudaEvent_t a0, a1;
    cudaEventCreate(&a0);
    cudaEventCreate(&a1);
    cudaGraphLaunch(ge, e->st);
    cudaEventRecord(a0, e->st);
    for (int i = 0; i < reps; ++i) cudaGraphLaunch(ge, e->st);
    cudaEventRecord(a1, e->st);
    cudaError_t se = cudaEventSynchronize(a1);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, a0, a1);
    cudaEventDestroy(a0);
    cudaEventDestroy(a1);
    cudaGraphExecDestroy(ge);
    cudaGraphDestroy(g);
    ALB_CUDA_TRY(se);
    *us_per_launch = ms * 1000.0f / (float)(reps * list.size());
    *ops_per_launch = ops / (double)list.size();
    return ALB_OK;
}

extern "C" int alb_engine_time_gemv(alb_engine * e, int32_t reps, float * us_per_launch, double * bytes_per_launch) {
    ALB_CHECK_ARG(e && reps > 0 && us_per_launch && bytes_per_launch);
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    std::vector<GemvArgs> list;
    double bytes = 0.0;
    // the decode step's mat-vec launches with the step's input modes (outputs to
    // scratch so the engine state is unchanged)
    auto add = [&](const uint8_t * W, int64_t N, int64_t K, int in, const void * x, const float * nw,
                   int out, float * y, const float * res) {
        GemvArgs a;
        a.W = W; a.N = N; a.K = K;
        a.in_mode = in; a.x = x; a.norm_w = nw; a.eps = e->c.eps;
        a.out_mode = out; a.y = y; a.residual = res; a.pdl = true;
        list.push_back(a);
        const double in_bytes = in == GEMV_IN_Q8 ? K / 32 * 34.0 : in == GEMV_IN_F32 ? K * 4.0 : K * 8.0;
        bytes += (double)N * K * 18 / 32 + in_bytes + (out == GEMV_OUT_SWIGLU ? N / 2 : N) * 4.0;
    };
    for (int l = 0; l < e->c.n_layer; ++l) {
        alb_engine::Layer & L = e->layers[l];
        add(L.qkv, e->Nqkv, e->E, GEMV_IN_F32_RMS, e->x, L.an, GEMV_OUT_PLAIN, e->qkv, nullptr);
        add(L.o, e->E, e->Dq, GEMV_IN_Q8, e->xq, nullptr, GEMV_OUT_PLAIN, e->qkv, nullptr);
        add(L.gu, 2 * (int64_t)e->F, e->E, GEMV_IN_F32_RMS, e->x, L.fn, GEMV_OUT_SWIGLU, e->h, nullptr);
        add(L.down, e->E, e->F, GEMV_IN_F32, e->h, nullptr, GEMV_OUT_PLAIN, e->qkv, nullptr);
    }
    add(e->lm_W, e->V, e->E, GEMV_IN_F32_RMS, e->x, e->out_norm, GEMV_OUT_PAIR, e->logits, nullptr);
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    ALB_CUDA_TRY(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal));
    cudaError_t le = cudaSuccess;
    for (const GemvArgs & a : list) if (le == cudaSuccess) le = launch_gemv(a, e->st);
    const cudaError_t ce = cudaStreamEndCapture(e->st, &g);
    ALB_CUDA_TRY(le);
    ALB_CUDA_TRY(ce);
    ALB_CUDA_TRY(cudaGraphInstantiate(&ge, g, 0));
    cudaEvent_t a0, a1;
    cudaEventCreate(&a0);
    cudaEventCreate(&a1);
    for (int i = 0; i < 2; ++i) cudaGraphLaunch(ge, e->st);
    cudaEventRecord(a0, e->st);
    for (int i = 0; i < reps; ++i) cudaGraphLaunch(ge, e->st);
    cudaEventRecord(a1, e->st);
    cudaError_t se = cudaEventSynchronize(a1);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, a0, a1);
    cudaEventDestroy(a0);
    cudaEventDestroy(a1);
    cudaGraphExecDestroy(ge);
    cudaGraphDestroy(g);
    ALB_CUDA_TRY(se);
    *us_per_launch = ms * 1000.0f / (float)(reps * list.size());
    *bytes_per_launch = bytes / (double)list.size();
    return ALB_OK;
}

// Config 5: fill the KV cache of every layer for positions [0, n_pos) with
// N(0,1) fp16 values (seeded per layer and K/V, indexed on the full KV row).
extern "C" int alb_engine_fill_kv(alb_engine * e, int32_t n_pos, uint64_t seed) {
    ALB_CHECK_ARG(e && n_pos > 0 && n_pos <= e->max_ctx);
    ALB_CUDA_TRY(cudaSetDevice(e->dev));
    const int64_t full = (int64_t)e->c.n_head_kv * e->c.head_dim;
    for (int l = 0; l < e->c.n_layer; ++l) {
        ALB_CUDA_TRY(gen_f16(e->layers[l].kc, n_pos, e->Dkv, full, (int64_t)e->rank * e->Dkv, tensor_seed(seed, l, 62),
                             e->table, e->st));
        ALB_CUDA_TRY(gen_f16(e->layers[l].vc, n_pos, e->Dkv, full, (int64_t)e->rank * e->Dkv, tensor_seed(seed, l, 63),
                             e->table, e->st));
    }
    ALB_CUDA_TRY(cudaStreamSynchronize(e->st));
    return ALB_OK;
}
