// al-bench: prefill a prompt and greedily decode with the B200 engine, reporting
// the reference driver's two performance lines.
//
// The counterpart of the reference's al-gen flow (apps/al-gen.cpp:13-141:
// load the model, build the KV cache and graph, ctx.infer(prompt, max_gen),
// ctx.print_perf()) over the C ABI of libalb_cuda.so.  The model is either a
// Qwen3 Q4_0 GGUF file (--gguf: configuration from its qwen3.* keys, tensors
// uploaded through alb_engine_set_weight_blocks / _set_norm_weights, each rank
// keeping its shard) or the seeded synthetic Qwen3 of a named shape (the engine
// generates it on the device).  There is no tokenizer: the prompt is seeded
// uniform token ids.  Tensor parallelism (--numa tp --nodes N in the
// reference, model.cpp:21-54) runs one thread per GPU rank, all ranks joining
// one NCCL clique.
//
//   al_bench [--model 0.6b|4b|8b|tiny|tiny_gqa | --gguf FILE] [--prompt N]
//            [--max_gen M] [--max_length L] [--ubatch U] [--seed S] [--nodes N]
//            [--loop] [--print_tokens]
#include <chrono>
#include <memory>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "alb_cuda.h"
#include "gguf_reader.h"

namespace {

struct Args {
    std::string model = "4b";
    std::string gguf_path;
    int prompt = 512, max_gen = 128, max_length = 0, ubatch = 256, nodes = 1;
    unsigned long long seed = 1234;
    bool loop = false, print_tokens = false;
};

bool config_of(const std::string & name, alb_qwen3_config & c) {
    // the shapes of arclight_b200/configs.py (Qwen3 model cards; tiny test shapes)
    if (name == "0.6b") c = {28, 1024, 16, 8, 128, 3072, 151936, 1, 1e-6f, 1e6f};
    else if (name == "4b") c = {36, 2560, 32, 8, 128, 9728, 151936, 1, 1e-6f, 1e6f};
    else if (name == "8b") c = {36, 4096, 32, 8, 128, 12288, 151936, 0, 1e-6f, 1e6f};
    else if (name == "tiny") c = {2, 512, 8, 8, 128, 1024, 4096, 1, 1e-6f, 1e6f};
    else if (name == "tiny_gqa") c = {3, 1024, 16, 4, 128, 2816, 8192, 0, 1e-6f, 1e6f};
    else return false;
    return true;
}

bool parse(int argc, char ** argv, Args & a) {
    for (int i = 1; i < argc; ++i) {
        const std::string k = argv[i];
        auto val = [&](const char * what) -> const char * {
            if (i + 1 >= argc) { std::fprintf(stderr, "al_bench: %s needs a value\n", what); std::exit(2); }
            return argv[++i];
        };
        if (k == "--model") a.model = val("--model");
        else if (k == "--gguf") a.gguf_path = val("--gguf");
        else if (k == "--prompt") a.prompt = std::atoi(val("--prompt"));
        else if (k == "--max_gen") a.max_gen = std::atoi(val("--max_gen"));
        else if (k == "--max_length") a.max_length = std::atoi(val("--max_length"));
        else if (k == "--ubatch") a.ubatch = std::atoi(val("--ubatch"));
        else if (k == "--seed") a.seed = std::strtoull(val("--seed"), nullptr, 10);
        else if (k == "--nodes") a.nodes = std::atoi(val("--nodes"));
        else if (k == "--loop") a.loop = true;
        else if (k == "--print_tokens") a.print_tokens = true;
        else { std::fprintf(stderr, "al_bench: unknown argument %s\n", k.c_str()); return false; }
    }
    if (a.max_length <= 0) a.max_length = a.prompt + a.max_gen + 8;
    return a.prompt > 0 && a.max_gen >= 0 && a.nodes >= 1 && a.max_length >= a.prompt + a.max_gen;
}

// Qwen3 configuration from a GGUF file's keys (models/qwen3.cpp:7-16).
bool config_from_gguf(const gguf::File & f, alb_qwen3_config & c) {
    const std::string & arch = f.str("general.architecture");
    if (!arch.empty() && arch != "qwen3") throw std::runtime_error("architecture " + arch + " is not qwen3");
    c.n_layer = (int32_t)f.num("qwen3.block_count");
    c.n_embd = (int32_t)f.num("qwen3.embedding_length");
    c.n_head = (int32_t)f.num("qwen3.attention.head_count");
    c.n_head_kv = (int32_t)f.num("qwen3.attention.head_count_kv");
    c.head_dim = (int32_t)f.num_or("qwen3.attention.key_length", c.n_embd / c.n_head);
    c.n_ff = (int32_t)f.num("qwen3.feed_forward_length");
    c.n_vocab = (int32_t)f.tensor("token_embd.weight").ne.at(1);
    c.tied = f.has_tensor("output.weight") ? 0 : 1;
    c.eps = (float)f.num_or("qwen3.attention.layer_norm_rms_epsilon", 1e-6);
    c.freq_base = (float)f.num_or("qwen3.rope.freq_base", 1e6);
    return true;
}

// Every tensor of the file into engine e (tensor names: models/qwen3.cpp:32-45;
// kinds: the C ABI's).
int upload_gguf(alb_engine * e, const gguf::File & f, const alb_qwen3_config & c) {
    struct Item { std::string name; int layer, kind; bool norm; };
    std::vector<Item> plan = {{"token_embd.weight", -1, 0, false}, {"output_norm.weight", -1, 2, true}};
    if (!c.tied) plan.push_back({"output.weight", -1, 1, false});
    const std::pair<const char *, int> per_layer[] = {
        {"attn_norm.weight", 3}, {"attn_q.weight", 4}, {"attn_k.weight", 5}, {"attn_v.weight", 6},
        {"attn_output.weight", 7}, {"attn_q_norm.weight", 8}, {"attn_k_norm.weight", 9}, {"ffn_norm.weight", 10},
        {"ffn_gate.weight", 11}, {"ffn_up.weight", 12}, {"ffn_down.weight", 13}};
    for (int l = 0; l < c.n_layer; ++l)
        for (const auto & [suffix, kind] : per_layer)
            plan.push_back({"blk." + std::to_string(l) + "." + suffix, l, kind, kind == 3 || kind == 8 || kind == 9 || kind == 10});
    for (const Item & it : plan) {
        const gguf::Tensor & t = f.tensor(it.name);
        int rc;
        if (it.norm) {
            int64_t n = 1;
            for (uint64_t x : t.ne) n *= (int64_t)x;
            std::vector<float> w((size_t)n);
            if (t.type == gguf::GGML_F32) std::memcpy(w.data(), f.data(t), (size_t)n * 4);
            else throw std::runtime_error(it.name + ": norm weights must be F32");
            rc = alb_engine_set_norm_weights(e, it.layer, it.kind, w.data(), n);
        } else {
            if (t.type != gguf::GGML_Q4_0 || t.ne.size() != 2) throw std::runtime_error(it.name + ": not a Q4_0 matrix");
            rc = alb_engine_set_weight_blocks(e, it.layer, it.kind, f.data(t), (int64_t)t.ne[1], (int64_t)t.ne[0]);
        }
        if (rc != ALB_OK) return rc;
    }
    return ALB_OK;
}

struct RankResult {
    int rc = ALB_OK;
    std::string what;
    double t_prefill_us = 0, t_decode_us = 0;
    std::vector<int32_t> tokens;
};

void run_rank(const Args & a, const alb_qwen3_config & cfg, const gguf::File * model, const std::vector<int32_t> & prompt,
              const void * nccl_id, int rank, RankResult & out) {
    alb_engine * e = nullptr;
    auto fail = [&](int rc, const char * what) {
        out.rc = rc;
        out.what = std::string(what) + ": " + alb_last_error();
    };
    int rc = alb_engine_create(&cfg, a.seed, a.max_length, a.ubatch, rank, a.nodes, nccl_id, rank, &e);
    if (rc != ALB_OK) { fail(rc, "alb_engine_create"); return; }
    if (model) {
        try {
            rc = upload_gguf(e, *model, cfg);
        } catch (const std::exception & x) {
            out.rc = ALB_ERR_INVALID;
            out.what = std::string("gguf: ") + x.what();
            alb_engine_destroy(e);
            return;
        }
        if (rc != ALB_OK) { fail(rc, "alb_engine_set_weight_blocks"); alb_engine_destroy(e); return; }
    }
    int32_t tok = 0;
    const auto t0 = std::chrono::steady_clock::now();
    rc = alb_engine_prefill(e, prompt.data(), (int32_t)prompt.size(), 0, &tok);
    const auto t1 = std::chrono::steady_clock::now();
    if (rc != ALB_OK) { fail(rc, "alb_engine_prefill"); alb_engine_destroy(e); return; }
    out.tokens.push_back(tok);
    const int32_t pos0 = (int32_t)prompt.size();
    if (a.loop && a.max_gen > 1) {
        // device-resident loop: token and position advance on the GPU
        std::vector<int32_t> gen((size_t)a.max_gen - 1);
        rc = alb_engine_decode_loop(e, tok, pos0, a.max_gen - 1, gen.data(), 1);
        if (rc == ALB_OK) out.tokens.insert(out.tokens.end(), gen.begin(), gen.end());
    } else {
        for (int i = 1; i < a.max_gen && rc == ALB_OK; ++i) {   // one call per token (decoding_context::infer)
            rc = alb_engine_decode(e, tok, pos0 + i - 1, &tok);
            out.tokens.push_back(tok);
        }
    }
    const auto t2 = std::chrono::steady_clock::now();
    if (rc != ALB_OK) fail(rc, "alb_engine_decode");
    out.t_prefill_us = std::chrono::duration<double, std::micro>(t1 - t0).count();
    out.t_decode_us = std::chrono::duration<double, std::micro>(t2 - t1).count();
    alb_engine_destroy(e);
}

}  // namespace

int main(int argc, char ** argv) {
    Args a;
    alb_qwen3_config cfg;
    std::unique_ptr<gguf::File> model;
    bool ok = parse(argc, argv, a);
    if (ok && !a.gguf_path.empty()) {
        try {
            model = std::make_unique<gguf::File>(a.gguf_path);
            config_from_gguf(*model, cfg);
        } catch (const std::exception & x) {
            std::fprintf(stderr, "al_bench: %s: %s\n", a.gguf_path.c_str(), x.what());
            return 1;
        }
    } else if (ok) {
        ok = config_of(a.model, cfg);
    }
    if (!ok) {
        std::fprintf(stderr, "usage: al_bench [--model 0.6b|4b|8b|tiny|tiny_gqa | --gguf FILE] [--prompt N] [--max_gen M] "
                             "[--max_length L] [--ubatch U] [--seed S] [--nodes N] [--loop] [--print_tokens]\n");
        return 2;
    }
    for (int r = 0; r < a.nodes; ++r) {
        if (alb_device_check(r) != ALB_OK) {
            std::fprintf(stderr, "al_bench: device %d: %s\n", r, alb_last_error());
            return 1;
        }
    }
    std::mt19937_64 rng(a.seed);
    std::vector<int32_t> prompt((size_t)a.prompt);
    for (auto & t : prompt) t = (int32_t)(rng() % (uint64_t)cfg.n_vocab);
    unsigned char nccl_id[128] = {0};
    if (a.nodes > 1 && alb_nccl_unique_id(nccl_id) != ALB_OK) {
        std::fprintf(stderr, "al_bench: %s\n", alb_last_error());
        return 1;
    }
    std::vector<RankResult> res((size_t)a.nodes);
    std::vector<std::thread> threads;
    for (int r = 0; r < a.nodes; ++r)
        threads.emplace_back(run_rank, std::cref(a), std::cref(cfg), model.get(), std::cref(prompt),
                             a.nodes > 1 ? (const void *)nccl_id : nullptr, r, std::ref(res[(size_t)r]));
    for (auto & t : threads) t.join();
    for (int r = 0; r < a.nodes; ++r) {
        if (res[(size_t)r].rc != ALB_OK) {
            std::fprintf(stderr, "al_bench: rank %d: %s\n", r, res[(size_t)r].what.c_str());
            return 1;
        }
        if (res[(size_t)r].tokens != res[0].tokens) {
            std::fprintf(stderr, "al_bench: rank %d generated different tokens than rank 0\n", r);
            return 1;
        }
    }
    const RankResult & r0 = res[0];
    if (a.print_tokens) {
        std::printf("prompt:");
        for (int32_t t : prompt) std::printf(" %d", t);
        std::printf("\ntokens:");
        for (int32_t t : r0.tokens) std::printf(" %d", t);
        std::printf("\n");
    }
    // the two lines of decoding_context::print_perf (context.cpp:245-255)
    const int n_pre = a.prompt, n_dec = (int)r0.tokens.size() - 1;
    std::printf("prefill time: %.2f ms / %4d token, %.2f ms/token, %.2f token/s\n", r0.t_prefill_us / 1000.0, n_pre,
                r0.t_prefill_us / 1000.0 / n_pre, n_pre * 1e6 / r0.t_prefill_us);
    if (n_dec > 0)
        std::printf("decode time:  %.2f ms / %4d token, %.2f ms/token, %.2f token/s\n", r0.t_decode_us / 1000.0, n_dec,
                    r0.t_decode_us / 1000.0 / n_dec, n_dec * 1e6 / r0.t_decode_us);
    return 0;
}
