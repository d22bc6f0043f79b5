// Driver for the reference's own KV-cache cell manager (oracle/_ref build only).
// Each refkv_* entry runs the reference's llm_kv_cache (nnml/src/cgraph.cpp:
// 915-1600, compiled from its own sources) on ubatches given as flat arrays,
// the same arguments as the alb_kv_* C ABI.  The cache is built with no layers
// (hparams.n_layer = 0), so it holds cells only and allocates no tensors; the
// mask is written through an nnml_tensor header over the caller's buffer.
// tests/golden/make_kv_golden.py calls these through ctypes to write the
// golden fixtures that pin alb_kvcache.cpp.  Test infrastructure only.
#include <algorithm>
#include <cstdint>
#include <vector>

#include "cgraph.h"
#include "tensor.h"

namespace {

// an llm_ubatch over flat (pos, seq) arrays: one sequence per token; the
// distinct sequence ids ascending, as the reference's batch allocator lists them
struct ub_store {
    std::vector<llm_pos> pos;
    std::vector<int32_t> n_seq_id;
    std::vector<llm_seq_id> seq;
    std::vector<llm_seq_id *> seq_ptr;
    std::vector<llm_seq_id> unq;
    llm_ubatch ub{};

    ub_store(const int32_t * p, const int32_t * s, int n) : pos(p, p + n), n_seq_id(n, 1), seq(s, s + n) {
        for (int i = 0; i < n; ++i) seq_ptr.push_back(&seq[i]);
        unq = seq;
        std::sort(unq.begin(), unq.end());
        unq.erase(std::unique(unq.begin(), unq.end()), unq.end());
        ub.b_equal_seqs = 1;
        ub.n_tokens = (uint32_t)n;
        ub.n_seqs_unq = (uint32_t)unq.size();
        ub.n_seqs = ub.n_seqs_unq;
        ub.n_seq_tokens = (uint32_t)n / ub.n_seqs_unq;
        ub.pos = pos.data();
        ub.n_seq_id = n_seq_id.data();
        ub.seq_id = seq_ptr.data();
        ub.seq_id_unq = unq.data();
    }
};

void put_idxs(const llm_kv_cache * kv, const llm_kv_cache::slot_info & si, int64_t * out) {
    const size_t sz = si.size();
    for (size_t s = 0; s < si.n_stream(); ++s)
        for (size_t k = 0; k < sz; ++k) out[s * sz + k] = (int64_t)si.strm[s] * kv->get_size() + si.idxs[s][k];
}

struct handle {
    llm_kv_cache * kv;
    uint32_t n_stream;
};

llm_kv_cache * K(void * h) { return static_cast<handle *>(h)->kv; }

}  // namespace

extern "C" {

void * refkv_create(uint32_t kv_size, uint32_t n_seq_max, int unified, uint32_t n_pad) {
    llm_hparams hp;
    hp.n_layer = 0;
    nnml_memory_t mem;   // not used: no layer, no tensor
    auto * kv = new llm_kv_cache(NNML_TYPE_F16, NNML_TYPE_F16, false, unified != 0, kv_size, n_seq_max, n_pad, hp, mem);
    return new handle{kv, unified ? 1u : n_seq_max};
}

void refkv_destroy(void * h) {
    delete K(h);
    delete static_cast<handle *>(h);
}

int refkv_find_slot(void * h, const int32_t * pos, const int32_t * seq, int n, int cont, int64_t * out) {
    ub_store u(pos, seq, n);
    const auto si = K(h)->find_slot(u.ub, cont != 0);
    if (si.empty()) return -7;
    put_idxs(K(h), si, out);
    return 0;
}

int refkv_prepare(void * h, const int32_t * sizes, int n_ub, const int32_t * pos, const int32_t * seq, int64_t * out) {
    std::vector<ub_store *> st;
    std::vector<llm_ubatch> ubs;
    int64_t off = 0;
    for (int b = 0; b < n_ub; ++b) {
        st.push_back(new ub_store(pos + off, seq + off, sizes[b]));
        ubs.push_back(st.back()->ub);
        off += sizes[b];
    }
    const auto res = K(h)->prepare(ubs);
    const int rc = res.empty() ? -7 : 0;
    off = 0;
    for (size_t b = 0; b < res.size(); ++b) {
        put_idxs(K(h), res[b], out + off);
        off += sizes[b];
    }
    for (auto * p : st) delete p;
    return rc;
}

// process_ubatch's kv->apply() (context.cpp:177-181) on the slot given as flat
// cell indices: one group per sequence run with several streams, else one
int refkv_apply(void * h, const int32_t * pos, const int32_t * seq, int n, const int64_t * idxs, uint32_t * n_kv) {
    llm_kv_cache * kv = K(h);
    ub_store u(pos, seq, n);
    const uint32_t size = kv->get_size();
    const uint32_t groups = static_cast<handle *>(h)->n_stream > 1 ? u.ub.n_seqs_unq : 1;
    const uint32_t sz = (uint32_t)n / groups;
    llm_kv_cache::slot_info si{};
    si.resize(groups);
    si.s0 = UINT32_MAX;
    si.s1 = 0;
    for (uint32_t s = 0; s < groups; ++s) {
        si.strm[s] = (llm_seq_id)(idxs[s * sz] / size);
        si.s0 = std::min<uint32_t>(si.s0, (uint32_t)si.strm[s]);
        si.s1 = std::max<uint32_t>(si.s1, (uint32_t)si.strm[s]);
        for (uint32_t k = 0; k < sz; ++k) si.idxs[s].push_back((uint32_t)(idxs[s * sz + k] % size));
    }
    kv->set_ubatchs({u.ub});
    kv->set_sinfos({si});
    kv->set_i_cur(0);
    kv->apply();
    *n_kv = kv->get_n_kv();
    return 0;
}

void refkv_seq_rm(void * h, int seq, int p0, int p1) { K(h)->seq_rm(seq, p0, p1); }

void refkv_seq_add(void * h, int seq, int p0, int p1, int shift) { K(h)->seq_add(seq, p0, p1, shift); }

void refkv_seq_pos_range(void * h, int seq, int32_t * mn, int32_t * mx) {
    *mn = K(h)->seq_pos_min(seq);
    *mx = K(h)->seq_pos_max(seq);
}

void refkv_mask(void * h, const int32_t * pos, const int32_t * seq, int n, int n_stream_ub, uint32_t n_kv,
                float * out) {
    ub_store u(pos, seq, n);
    const int64_t n_tps_pad = NNML_PAD((int64_t)(n / n_stream_ub), NNML_KQ_MASK_PAD);
    // a tensor header over `out`, allocated per call and not freed (these
    // sources declare nnml_tensor's destructor without defining it)
    nnml_tensor * t = new nnml_tensor();
    t->set_elements(0, n_kv);
    t->set_elements(1, n_tps_pad);
    t->set_elements(2, 1);
    t->set_elements(3, n_stream_ub);
    t->set_tensor_data(out);
    K(h)->set_kq_mask(t, 0);
    K(h)->set_inputs_attn_mask(&u.ub);
    K(h)->set_kq_mask(nullptr, 0);
}

}  // extern "C"
