"""Write tests/golden/kv_cache_golden.json.gz: seeded KV-cache operation scripts
run on the reference's own llm_kv_cache (oracle/_ref/libalref.so, built by
`make -C oracle ref REF=<reference tree>`), every call with its result.
tests/test_kvcache.py replays them on alb_kv_* and requires identical results.

    python tests/golden/make_kv_golden.py
"""
import gzip
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.kv_script import CONFIGS, RefBackend, record  # noqa: E402

SEEDS = (11, 12)
N_OPS = 120


def main() -> None:
    if not RefBackend.available():
        sys.exit("oracle/_ref/libalref.so is not built (make -C oracle ref REF=<reference tree>)")
    scripts = []
    for cfg in CONFIGS:
        for seed in SEEDS:
            scripts.append({"config": list(cfg), "seed": seed, "ops": record(cfg, seed, N_OPS, RefBackend(cfg))})
    out = os.path.join(HERE, "kv_cache_golden.json.gz")
    with gzip.open(out, "wt") as f:
        json.dump({"source": "reference llm_kv_cache (nnml/src/cgraph.cpp) via oracle/ref_kv_driver.cpp",
                   "scripts": scripts}, f, separators=(",", ":"))
    print("wrote", out, os.path.getsize(out), "bytes,", sum(len(s["ops"]) for s in scripts), "calls")


if __name__ == "__main__":
    main()
