// Parameters of the persistent decode-step kernel (alb_decode_mk.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace alb {

struct MkLayer {
    const uint8_t * qkv_W, * qkv_S, * o_W, * o_S, * gu_W, * gu_S, * dn_W, * dn_S;   // alb Q4_0 planes
    const float * an, * fn, * qn, * kn;                                              // norm weights
    uint16_t * kc, * vc;                                                             // [cells][Hkv][128] fp16
};

// Most cells one attention split of the persistent kernel handles (its scores
// live in shared memory); the engine uses the kernel only below this bound.
constexpr int MK_ATT_MAX_CELLS = 384;
// Byte offset in the shared union above which the attention inputs are staged
// while the QKV phase's Q8_0 records (48 bytes per 32 values of n_embd) sit
// below it: the kernel needs n_embd / 32 * 48 <= MK_STAGE_OFFSET.
constexpr int MK_STAGE_OFFSET = 4 * MK_ATT_MAX_CELLS * 8;

struct MkParams {
    int n_layer, E, Hq, Hkv, F, V, Nqkv, Dq, v0, rank;
    float eps, scale;
    int pf_stages;                   // stages the producer prefetches into L2 ahead of its copies
    const MkLayer * layers;          // device array [n_layer]
    const uint8_t * lm_W, * lm_S;    // lm head shard (rows [v0, v0 + V))
    const float * out_norm;
    const uint8_t * tok_W, * tok_S;  // full token table (embedding)
    const float * rope;              // [max_pos][64] (cos, sin)
    float * x, * qkv, * att, * h, * logits;
    int32_t * tok, * pos, * next, * gen_out, * step;
    int gen_cap, advance;
    int S;                           // attention splits (Hkv * S <= ncta)
    float * smax;                    // [Hkv][S][G]
    double * part;                   // [Hkv][S][8][G][129]
    unsigned * grp;                  // [Hkv][2] per-head barrier count / generation, zero at first use
    int * tickets;                   // [Hkv], zero at first use
    unsigned long long * cand;       // [ncta]
    int * am_ticket;                 // zero at first use
    unsigned * bar_count, * bar_gen; // grid barrier words, zero at first use
    int * err;
    int64_t * trace;                 // nullable: CTA 0 records %globaltimer at phase boundaries
    int ncta;
};

size_t mk_smem_bytes();
cudaError_t launch_decode_step(const MkParams & p, cudaStream_t st);

}  // namespace alb
