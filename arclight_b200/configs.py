"""Qwen3 shapes of the benchmark configs and a tiny test shape."""

QWEN3_0_6B = dict(n_layer=28, n_embd=1024, n_head=16, n_head_kv=8, head_dim=128, n_ff=3072, n_vocab=151936,
                  tied=1, eps=1e-6, freq_base=1e6)
QWEN3_4B = dict(n_layer=36, n_embd=2560, n_head=32, n_head_kv=8, head_dim=128, n_ff=9728, n_vocab=151936,
                tied=1, eps=1e-6, freq_base=1e6)
QWEN3_8B = dict(n_layer=36, n_embd=4096, n_head=32, n_head_kv=8, head_dim=128, n_ff=12288, n_vocab=151936,
                tied=0, eps=1e-6, freq_base=1e6)
# small model with the Qwen3 structure for fast parity tests (8 heads so TP up to 8 divides)
TINY = dict(n_layer=2, n_embd=512, n_head=8, n_head_kv=8, head_dim=128, n_ff=1024, n_vocab=4096,
            tied=1, eps=1e-6, freq_base=1e6)
TINY_GQA = dict(n_layer=3, n_embd=1024, n_head=16, n_head_kv=4, head_dim=128, n_ff=2816, n_vocab=8192,
                tied=0, eps=1e-6, freq_base=1e6)

CONFIGS = {"0.6b": QWEN3_0_6B, "4b": QWEN3_4B, "8b": QWEN3_8B, "tiny": TINY, "tiny_gqa": TINY_GQA}
