// KV-cache cell manager (host): slot search, placement, sequence removal and
// shifts, padded KV length and the attention mask of the reference's
// llm_kv_cache / llm_kv_cells (nnml/include/cgraph.h:249-374, 612-1046;
// nnml/src/cgraph.cpp:915-1600).  The search and the bookkeeping follow the
// reference step by step -- the cell every token lands in decides where its
// K/V row is stored and which rows each query sees, so it has to be the same
// cell -- in a layout of its own: one 64-bit sequence mask per cell and, per
// sequence, a count of cells at each position.
//
// For one sequence prefilled and decoded in position order (al-gen's use), and
// after a truncation by seq_rm(seq, p, -1) that is then refilled from p, cell c
// holds position c: the engine's device cache is addressed by position for that
// reason, and the KV-cache tests check this property.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <limits>
#include <map>
#include <new>
#include <set>
#include <vector>

#include "alb_kvcache.h"

void alb_set_last_error_msg(const char * msg);

namespace {

constexpr int MAX_SEQ = ALB_KV_MAX_SEQ;

// NNML_PAD (nnml.h:115), for the power-of-two paddings the cache uses
inline uint32_t pad_up(uint32_t x, uint32_t n) { return (x + n - 1) & ~(n - 1); }

// The cells of one stream (llm_kv_cells, cgraph.h:612-1046).
struct Cells {
    std::vector<int32_t> pos;       // -1: empty
    std::vector<int32_t> shift;     // accumulated seq_add shift of the cell
    std::vector<uint64_t> seqs;     // bit s: sequence s holds the cell
    std::set<uint32_t> used;        // non-empty cells, ordered
    std::map<int32_t, int32_t> at[MAX_SEQ];   // per sequence: position -> cells holding it
    bool has_shift = false;

    void init(uint32_t n) {
        pos.assign(n, -1);
        shift.assign(n, 0);
        seqs.assign(n, 0);
        used.clear();
        for (auto & m : at) m.clear();
        has_shift = false;
    }
    uint32_t size() const { return (uint32_t)pos.size(); }
    bool empty(uint32_t i) const { return pos[i] == -1; }
    bool has(uint32_t i, int s) const { return (seqs[i] >> s) & 1u; }
    bool pos_in(uint32_t i, int32_t p0, int32_t p1) const { return pos[i] >= p0 && pos[i] < p1; }
    uint32_t used_max_p1() const { return used.empty() ? 0u : *used.rbegin() + 1u; }

    void count(int s, int32_t p, int d) {
        auto & m = at[s];
        if (d > 0) {
            ++m[p];
        } else {
            auto it = m.find(p);
            if (it != m.end() && --it->second == 0) m.erase(it);
        }
    }
    // add (+1) or withdraw (-1) every (sequence, position) pair of cell i
    void count_cell(uint32_t i, int d) {
        for (uint64_t b = seqs[i]; b; b &= b - 1) count(__builtin_ctzll(b), pos[i], d);
    }
    void free_cell(uint32_t i) {
        pos[i] = -1;
        shift[i] = 0;
        seqs[i] = 0;
        used.erase(i);
    }
    void rm(uint32_t i) {   // llm_kv_cells::rm
        count_cell(i, -1);
        free_cell(i);
    }
    bool seq_rm(uint32_t i, int s) {   // llm_kv_cells::seq_rm: true if the cell became empty
        seqs[i] &= ~(1ull << s);
        count(s, pos[i], -1);
        if (seqs[i] == 0) {
            free_cell(i);
            return true;
        }
        return false;
    }
    void seq_add(uint32_t i, int s) {   // llm_kv_cells::seq_add
        seqs[i] |= 1ull << s;
        count(s, pos[i], +1);
    }
    void pos_set(uint32_t i, int32_t p) {   // llm_kv_cells::pos_set on an empty cell
        pos[i] = p;
        used.insert(i);
    }
    bool pos_add(uint32_t i, int32_t d) {   // llm_kv_cells::pos_add: true if the cell was freed
        count_cell(i, -1);
        pos[i] += d;
        shift[i] += d;
        has_shift = true;
        if (pos[i] < 0) {
            free_cell(i);
            return true;
        }
        count_cell(i, +1);
        return false;
    }
    int32_t pos_min(int s) const { return at[s].empty() ? -1 : at[s].begin()->first; }
    int32_t pos_max(int s) const { return at[s].empty() ? -1 : at[s].rbegin()->first; }

    // llm_kv_cells::cp / set over a list of cells (positions and sequences; shifts untouched)
    struct Saved {
        std::vector<int32_t> pos;
        std::vector<uint64_t> seqs;
    };
    Saved save(const std::vector<uint32_t> & idx) const {
        Saved s;
        for (uint32_t i : idx) {
            s.pos.push_back(pos[i]);
            s.seqs.push_back(seqs[i]);
        }
        return s;
    }
    void restore(const std::vector<uint32_t> & idx, const Saved & s) {
        for (size_t j = 0; j < idx.size(); ++j) {
            const uint32_t i = idx[j];
            if (pos[i] == -1 && s.pos[j] != -1) used.insert(i);
            if (pos[i] != -1 && s.pos[j] == -1) used.erase(i);
            if (pos[i] != -1) count_cell(i, -1);
            pos[i] = s.pos[j];
            seqs[i] = s.seqs[j];
            if (pos[i] != -1) count_cell(i, +1);
        }
    }
};

// llm_kv_cache::slot_info: per sequence group of the ubatch, its stream and cells
struct Slot {
    std::vector<uint32_t> strm;
    std::vector<std::vector<uint32_t>> idxs;
    bool empty() const { return idxs.empty(); }
    size_t size() const { return idxs[0].size(); }
};

// One ubatch: n tokens, one sequence each; unq = its sequence ids, ascending.
struct Ubatch {
    int32_t n = 0;
    const int32_t * pos = nullptr;
    const int32_t * seq = nullptr;
    std::vector<int32_t> unq;
};

}  // namespace

struct alb_kv_cache {
    uint32_t size = 0, n_pad = 0, n_seq_max = 0, n_stream = 0;
    uint32_t n_kv = 0;
    std::vector<Cells> cells;              // [n_stream]
    std::vector<uint32_t> head;            // [n_stream]: where the next search starts
    std::vector<uint32_t> seq_to_stream;   // [64] (one stream) or [n_seq_max]
};

namespace {

int fail(int code, const char * msg) {
    alb_set_last_error_msg(msg);
    return code;
}

// Build the ubatch view and check it against the cache (sequence ids in range;
// with several streams, equal runs of one sequence each, in ascending order).
int make_ubatch(const alb_kv_cache * kv, const int32_t * pos, const int32_t * seq, int32_t n, Ubatch & u) {
    if (!kv || !pos || !seq || n <= 0) return fail(ALB_ERR_INVALID, "kv: bad ubatch arguments");
    u.n = n;
    u.pos = pos;
    u.seq = seq;
    uint64_t present = 0;
    for (int32_t i = 0; i < n; ++i) {
        if (seq[i] < 0 || seq[i] >= (int32_t)kv->seq_to_stream.size())
            return fail(ALB_ERR_INVALID, "kv: sequence id out of range");
        if (pos[i] < 0) return fail(ALB_ERR_INVALID, "kv: negative position");
        present |= 1ull << seq[i];
    }
    u.unq.clear();
    for (int s = 0; s < MAX_SEQ; ++s)
        if ((present >> s) & 1u) u.unq.push_back(s);
    if (kv->n_stream > 1) {
        const int32_t ns = (int32_t)u.unq.size();
        if (n % ns != 0) return fail(ALB_ERR_INVALID, "kv: tokens are not equal runs per sequence");
        const int32_t run = n / ns;
        for (int32_t i = 0; i < n; ++i)
            if (seq[i] != u.unq[i / run]) return fail(ALB_ERR_INVALID, "kv: tokens are not equal runs per sequence");
    }
    return ALB_OK;
}

// llm_kv_cache::find_slot (cgraph.cpp:1317-1418)
int find_slot(const alb_kv_cache * kv, const Ubatch & u, bool cont, Slot & res) {
    uint32_t n_tokens = (uint32_t)u.n, n_seqs = 1;
    if (kv->n_stream > 1) {
        n_seqs = (uint32_t)u.unq.size();
        n_tokens /= n_seqs;
    }
    res.strm.assign(n_seqs, 0);
    res.idxs.assign(n_seqs, {});
    for (uint32_t s = 0; s < n_seqs; ++s) {
        const uint32_t st = kv->seq_to_stream[u.unq[s]];
        res.strm[s] = st;
        const Cells & c = kv->cells[st];
        auto & out = res.idxs[s];
        out.reserve(n_tokens);
        uint32_t h = kv->head[st];
        // many free cells before the head: search from the start, to fill the cache
        if (h > (uint32_t)c.used.size() + 2 * n_tokens) h = 0;
        if (n_tokens > c.size()) return fail(ALB_ERR_INVALID, "kv: ubatch larger than the cache");
        const uint32_t n_test = cont ? n_tokens : 1;
        uint32_t n_tested = 0;
        while (true) {
            if (h + n_test > c.size()) {   // wrap to the start
                n_tested += c.size() - h;
                h = 0;
                continue;
            }
            for (uint32_t k = 0; k < n_test; ++k) {
                const uint32_t idx = h++;
                ++n_tested;
                if (c.empty(idx)) {
                    out.push_back(idx);
                } else if (cont) {
                    break;
                }
            }
            if (out.size() == n_tokens) break;
            if (cont) out.clear();
            if (n_tested >= c.size()) {
                res = Slot{};
                return ALB_ERR_NO_SLOT;
            }
        }
    }
    return ALB_OK;
}

// llm_kv_cache::seq_rm (cgraph.cpp:1535-1592)
void seq_rm(alb_kv_cache * kv, int32_t sid, int32_t p0, int32_t p1) {
    if (p0 < 0) p0 = 0;
    if (p1 < 0) p1 = std::numeric_limits<int32_t>::max();
    auto sweep = [&](uint32_t st, bool any_seq) {
        Cells & c = kv->cells[st];
        uint32_t & h = kv->head[st];
        uint32_t new_head = c.size();
        for (uint32_t i = 0; i < c.size(); ++i) {
            if (!c.pos_in(i, p0, p1)) continue;
            bool freed;
            if (any_seq) {
                c.rm(i);
                freed = true;
            } else {
                freed = c.has(i, sid) && c.seq_rm(i, sid);
            }
            if (freed && new_head == c.size()) new_head = i;
        }
        // a freed cell before the head: the next search starts there
        if (new_head != c.size() && new_head < h) h = new_head;
    };
    if (sid >= 0) {
        sweep(kv->seq_to_stream[sid], false);
    } else {
        for (uint32_t st = 0; st < kv->n_stream; ++st) sweep(st, true);
    }
}

// llm_kv_cache::apply_ubatch (cgraph.cpp:1420-1468)
int apply_ubatch(alb_kv_cache * kv, const Slot & sl, const Ubatch & u) {
    const size_t sz = sl.size();
    // the reference asserts this; here it is checked before any cell changes
    for (size_t s = 0; s < sl.strm.size(); ++s)
        for (uint32_t idx : sl.idxs[s]) {
            const Cells & c = kv->cells[sl.strm[s]];
            if (!c.empty(idx) && __builtin_popcountll(c.seqs[idx]) != 1)
                return fail(ALB_ERR_INVALID, "kv: overwritten cell is not held by exactly one sequence");
        }
    int32_t max_rm[MAX_SEQ];   // highest position overwritten per sequence
    for (auto & m : max_rm) m = -1;
    for (size_t s = 0; s < sl.strm.size(); ++s) {
        Cells & c = kv->cells[sl.strm[s]];
        for (size_t k = 0; k < sz; ++k) {
            const size_t i = s * sz + k;
            const uint32_t idx = sl.idxs[s][k];
            if (!c.empty(idx)) {
                const int prev = __builtin_ctzll(c.seqs[idx]);
                if (c.pos[idx] > max_rm[prev]) max_rm[prev] = c.pos[idx];
                c.rm(idx);
            }
            c.pos_set(idx, u.pos[i]);
            c.seq_add(idx, u.seq[i]);
        }
    }
    // a sequence that lost cells loses every position up to the last one lost
    for (int s = 0; s < MAX_SEQ; ++s) {
        if (max_rm[s] == -1) continue;
        const Cells & c = kv->cells[kv->seq_to_stream[s]];
        if (c.pos_min(s) <= max_rm[s]) seq_rm(kv, s, c.pos_min(s), max_rm[s] + 1);
    }
    for (size_t s = 0; s < sl.strm.size(); ++s) kv->head[sl.strm[s]] = sl.idxs[s].back() + 1;
    return ALB_OK;
}

// llm_kv_cache::get_n_kv (cgraph.cpp:1475-1482)
uint32_t get_n_kv(const alb_kv_cache * kv, const Slot & sl) {
    uint32_t r = 0;
    for (uint32_t st : sl.strm) {
        const Cells & c = kv->cells[st];
        const uint32_t want = std::max(kv->n_pad, pad_up(c.used_max_p1(), kv->n_pad));
        r = std::max(r, std::min(c.size(), want));
    }
    return r;
}

void write_idxs(const alb_kv_cache * kv, const Slot & sl, int64_t * out) {
    const size_t sz = sl.size();
    for (size_t s = 0; s < sl.strm.size(); ++s)
        for (size_t k = 0; k < sz; ++k) out[s * sz + k] = (int64_t)sl.strm[s] * kv->size + sl.idxs[s][k];
}

}  // namespace

extern "C" {

int alb_kv_create(uint32_t kv_size, uint32_t n_seq_max, int32_t unified, uint32_t n_pad, alb_kv_cache ** out) {
    if (!out) return fail(ALB_ERR_INVALID, "kv: null handle");
    *out = nullptr;
    if (kv_size == 0 || n_pad == 0 || kv_size % n_pad != 0 || n_seq_max == 0 || n_seq_max > MAX_SEQ)
        return fail(ALB_ERR_INVALID, "kv: bad cache shape");
    alb_kv_cache * kv = new (std::nothrow) alb_kv_cache;
    if (!kv) return fail(ALB_ERR_OOM, "kv: out of host memory");
    kv->size = kv_size;
    kv->n_pad = n_pad;
    kv->n_seq_max = n_seq_max;
    kv->n_stream = unified ? 1u : n_seq_max;
    kv->cells.resize(kv->n_stream);
    for (auto & c : kv->cells) c.init(kv_size);
    kv->head.assign(kv->n_stream, 0);
    // every sequence in stream 0, or sequence s in stream s (one per sequence)
    if (kv->n_stream > 1) {
        for (uint32_t s = 0; s < kv->n_stream; ++s) kv->seq_to_stream.push_back(s);
    } else {
        kv->seq_to_stream.assign(MAX_SEQ, 0);
    }
    *out = kv;
    return ALB_OK;
}

int alb_kv_destroy(alb_kv_cache * kv) {
    delete kv;
    return ALB_OK;
}

int alb_kv_clear(alb_kv_cache * kv) {
    if (!kv) return fail(ALB_ERR_INVALID, "kv: null handle");
    for (auto & c : kv->cells) c.init(kv->size);
    for (auto & h : kv->head) h = 0;
    return ALB_OK;
}

int alb_kv_find_slot(const alb_kv_cache * kv, const int32_t * pos, const int32_t * seq_id, int32_t n_tokens,
                     int32_t cont, int64_t * idxs_out) {
    Ubatch u;
    int r = make_ubatch(kv, pos, seq_id, n_tokens, u);
    if (r != ALB_OK) return r;
    if (!idxs_out) return fail(ALB_ERR_INVALID, "kv: null output");
    Slot sl;
    r = find_slot(kv, u, cont != 0, sl);
    if (r != ALB_OK) return r;
    write_idxs(kv, sl, idxs_out);
    return ALB_OK;
}

int alb_kv_prepare(alb_kv_cache * kv, const int32_t * sizes, int32_t n_ubatches, const int32_t * pos,
                   const int32_t * seq_id, int64_t * idxs_out) {
    if (!kv || !sizes || n_ubatches <= 0 || !idxs_out) return fail(ALB_ERR_INVALID, "kv: bad prepare arguments");
    std::vector<Ubatch> ubs(n_ubatches);
    int64_t off = 0;
    for (int32_t b = 0; b < n_ubatches; ++b) {
        const int r = make_ubatch(kv, pos + off, seq_id + off, sizes[b], ubs[b]);
        if (r != ALB_OK) return r;
        off += sizes[b];
    }
    struct State {
        Slot slot;
        std::vector<uint32_t> heads_old;
        std::vector<Cells::Saved> saved;
    };
    std::vector<Slot> res;
    std::vector<State> states;
    int status = ALB_OK;
    for (const Ubatch & u : ubs) {
        Slot sl;
        status = find_slot(kv, u, false, sl);
        if (status != ALB_OK) break;
        State st{sl, kv->head, {}};
        for (size_t s = 0; s < sl.strm.size(); ++s) st.saved.push_back(kv->cells[sl.strm[s]].save(sl.idxs[s]));
        states.push_back(std::move(st));
        res.push_back(sl);
        status = apply_ubatch(kv, sl, u);
        if (status != ALB_OK) break;
    }
    // undo the placements, last first (the saved heads are taken by the slot's
    // group index, as llm_kv_cache::prepare restores them)
    for (auto it = states.rbegin(); it != states.rend(); ++it) {
        for (size_t s = 0; s < it->slot.strm.size(); ++s) {
            kv->cells[it->slot.strm[s]].restore(it->slot.idxs[s], it->saved[s]);
            kv->head[it->slot.strm[s]] = it->heads_old[s];
        }
    }
    if (status != ALB_OK) return status;
    off = 0;
    for (size_t b = 0; b < res.size(); ++b) {
        write_idxs(kv, res[b], idxs_out + off);
        off += sizes[b];
    }
    return ALB_OK;
}

int alb_kv_apply(alb_kv_cache * kv, const int32_t * pos, const int32_t * seq_id, int32_t n_tokens,
                 const int64_t * idxs, uint32_t * n_kv_out) {
    Ubatch u;
    int r = make_ubatch(kv, pos, seq_id, n_tokens, u);
    if (r != ALB_OK) return r;
    if (!idxs) return fail(ALB_ERR_INVALID, "kv: null cell indices");
    const uint32_t n_seqs = kv->n_stream > 1 ? (uint32_t)u.unq.size() : 1u;
    const uint32_t sz = (uint32_t)n_tokens / n_seqs;
    Slot sl;
    sl.strm.assign(n_seqs, 0);
    sl.idxs.assign(n_seqs, {});
    for (uint32_t s = 0; s < n_seqs; ++s) {
        for (uint32_t k = 0; k < sz; ++k) {
            const int64_t f = idxs[s * sz + k];
            if (f < 0 || f >= (int64_t)kv->n_stream * kv->size) return fail(ALB_ERR_INVALID, "kv: cell index out of range");
            const uint32_t st = (uint32_t)(f / kv->size);
            if (k == 0) sl.strm[s] = st;
            if (st != sl.strm[s]) return fail(ALB_ERR_INVALID, "kv: one sequence's cells span streams");
            sl.idxs[s].push_back((uint32_t)(f % kv->size));
        }
    }
    std::vector<int64_t> sorted(idxs, idxs + n_tokens);   // no cell twice
    std::sort(sorted.begin(), sorted.end());
    if (std::adjacent_find(sorted.begin(), sorted.end()) != sorted.end())
        return fail(ALB_ERR_INVALID, "kv: a cell given twice");
    r = apply_ubatch(kv, sl, u);
    if (r != ALB_OK) return r;
    kv->n_kv = get_n_kv(kv, sl);
    if (n_kv_out) *n_kv_out = kv->n_kv;
    return ALB_OK;
}

int alb_kv_seq_rm(alb_kv_cache * kv, int32_t seq_id, int32_t p0, int32_t p1) {
    if (!kv || seq_id < -1 || seq_id >= (int32_t)kv->seq_to_stream.size())
        return fail(ALB_ERR_INVALID, "kv: bad seq_rm arguments");
    seq_rm(kv, seq_id, p0, p1);
    return ALB_OK;
}

int alb_kv_seq_add(alb_kv_cache * kv, int32_t seq_id, int32_t p0, int32_t p1, int32_t shift) {
    if (!kv || seq_id < 0 || seq_id >= (int32_t)kv->seq_to_stream.size())
        return fail(ALB_ERR_INVALID, "kv: bad seq_add arguments");
    const uint32_t st = kv->seq_to_stream[seq_id];
    Cells & c = kv->cells[st];
    if (shift == 0) return ALB_OK;
    if (p0 < 0) p0 = 0;
    if (p1 < 0) p1 = std::numeric_limits<int32_t>::max();
    if (p0 == p1) return ALB_OK;
    uint32_t new_head = c.size();
    for (uint32_t i = 0; i < c.size(); ++i) {
        if (!c.pos_in(i, p0, p1) || !c.has(i, seq_id)) continue;
        if (c.pos_add(i, shift) && new_head == c.size()) new_head = i;
    }
    // the first freed cell, else the start
    kv->head[st] = new_head != c.size() ? new_head : 0;
    return ALB_OK;
}

int alb_kv_seq_pos_range(const alb_kv_cache * kv, int32_t seq_id, int32_t * pos_min, int32_t * pos_max) {
    if (!kv || seq_id < 0 || seq_id >= (int32_t)kv->seq_to_stream.size())
        return fail(ALB_ERR_INVALID, "kv: bad sequence id");
    const Cells & c = kv->cells[kv->seq_to_stream[seq_id]];
    if (pos_min) *pos_min = c.pos_min(seq_id);
    if (pos_max) *pos_max = c.pos_max(seq_id);
    return ALB_OK;
}

int alb_kv_mask(const alb_kv_cache * kv, const int32_t * pos, const int32_t * seq_id, int32_t n_tokens,
                int32_t n_stream_ub, uint32_t n_kv, float * mask) {
    Ubatch u;
    int r = make_ubatch(kv, pos, seq_id, n_tokens, u);
    if (r != ALB_OK) return r;
    if (!mask || n_stream_ub <= 0 || n_tokens % n_stream_ub != 0 || n_kv == 0 || n_kv > kv->size)
        return fail(ALB_ERR_INVALID, "kv: bad mask arguments");
    const uint32_t n_tps = (uint32_t)(n_tokens / n_stream_ub);
    const uint32_t n_tps_pad = pad_up(n_tps, ALB_KV_MASK_PAD);
    const float ninf = -std::numeric_limits<float>::infinity();
    const size_t total = (size_t)n_stream_ub * n_tps_pad * n_kv;
    for (size_t i = 0; i < total; ++i) mask[i] = ninf;
    for (uint32_t s = 0; s < (uint32_t)n_stream_ub; ++s) {
        for (uint32_t k = 0; k < n_tps; ++k) {
            const uint32_t i = s * n_tps + k;
            const int sid = u.seq[i];
            const Cells & c = kv->cells[kv->seq_to_stream[sid]];
            const int32_t p1 = u.pos[i];
            float * row = mask + (size_t)n_kv * (s * n_tps_pad + k);
            for (uint32_t j = 0; j < n_kv; ++j)
                if (!c.empty(j) && c.has(j, sid) && c.pos[j] <= p1) row[j] = 0.0f;
        }
    }
    return ALB_OK;
}

int alb_kv_visible_cells(const alb_kv_cache * kv, int32_t seq_id, int32_t pos, uint32_t n_kv, int64_t * cells_out,
                         int32_t * n_out) {
    if (!kv || !cells_out || !n_out || seq_id < 0 || seq_id >= (int32_t)kv->seq_to_stream.size() || n_kv == 0 ||
        n_kv > kv->size)
        return fail(ALB_ERR_INVALID, "kv: bad visible-cells arguments");
    const uint32_t st = kv->seq_to_stream[seq_id];
    const Cells & c = kv->cells[st];
    int32_t n = 0;
    for (uint32_t j = 0; j < n_kv; ++j)
        if (!c.empty(j) && c.has(j, seq_id) && c.pos[j] <= pos) cells_out[n++] = (int64_t)st * kv->size + j;
    *n_out = n;
    return ALB_OK;
}

int alb_kv_cell(const alb_kv_cache * kv, uint32_t stream, uint32_t cell, int32_t * pos, uint64_t * seqs,
                int32_t * shift) {
    if (!kv || stream >= kv->n_stream || cell >= kv->size) return fail(ALB_ERR_INVALID, "kv: bad cell");
    const Cells & c = kv->cells[stream];
    if (pos) *pos = c.pos[cell];
    if (seqs) *seqs = c.seqs[cell];
    if (shift) *shift = c.shift[cell];
    return ALB_OK;
}

int alb_kv_info(const alb_kv_cache * kv, uint32_t stream, int64_t * info, int32_t n) {
    if (!kv || !info || stream >= kv->n_stream) return fail(ALB_ERR_INVALID, "kv: bad info arguments");
    const Cells & c = kv->cells[stream];
    const int64_t v[6] = {kv->size, kv->n_stream, kv->n_pad, (int64_t)c.used.size(), kv->head[stream],
                          c.used_max_p1()};
    for (int32_t i = 0; i < n && i < 6; ++i) info[i] = v[i];
    return ALB_OK;
}

}  // extern "C"
