#!/usr/bin/env python3
"""Generates the oracle fixtures of the full-depth model configurations.

The strict oracle build (oracle/, the CPU restatement of
src/transformer.cpp:128-243) decodes the seeded synthetic model that the
library's aaedn_model_synthesize builds (same generator and quantizer,
checked bit for bit by tests/test_oracle_golden.py) and the fixture keeps
what the GPU tests and bench.py compare against:

  llama2_7b_seed1234.npz  Llama-2-7B shape (dim 4096, 32 layers, 32 heads x
                          128, ffn 11008, vocab 32000, theta 10000), seed
                          1234: the 128-token prompt (stream 0), the first 64
                          greedy tokens after it, the logits after the prompt
                          and after the 64th token's step.

A full-depth 7B decode takes the oracle tens of minutes on a few cores, so
the GPU side reads these files instead of running the oracle itself.

    python tests/golden/make_model_fixtures.py [--threads N] [--only NAME]
"""
import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import pyoracle  # noqa: E402

LLAMA2_7B = dict(dim=4096, n_layers=32, n_heads=32, n_kv_heads=32, head_dim=128, ffn_dim=11008, vocab=32000,
                 max_seq=256, rope_theta=10000.0, eps=1e-6)

FIXTURES = {
    # name: (config, seed, prompt length, greedy tokens)
    "llama2_7b_seed1234": (LLAMA2_7B, 1234, 128, 64),
}


def make(name, threads):
    cfg, seed, n_prompt, n_new = FIXTURES[name]
    o = pyoracle.Oracle()
    if threads:
        o.set_threads(threads)
    t0 = time.time()
    w = pyoracle.synthetic_weights(cfg, seed, o)
    prompt = o.synth_tokens(seed, 0, cfg["vocab"], n_prompt)
    print(f"{name}: weights in {time.time() - t0:.0f} s", flush=True)
    om = pyoracle.OracleModel(o, cfg, w)
    t0 = time.time()
    logits = None
    for t in prompt:
        logits = om.step(int(t))
    logits_prompt = logits.copy()
    tokens = np.empty(n_new, np.uint32)
    for i in range(n_new):
        tokens[i] = int(np.argmax(logits))  # greedy, ties to the lowest id (D8)
        if i + 1 < n_new:
            logits = om.step(int(tokens[i]))
    print(f"{name}: {n_prompt + n_new - 1} steps in {time.time() - t0:.0f} s", flush=True)
    out = os.path.join(HERE, name + ".npz")
    np.savez_compressed(out, prompt=prompt, tokens=tokens, logits_prompt=logits_prompt, logits_last=logits,
                        seed=np.array(seed), config=np.array(repr(sorted(cfg.items()))))
    print("wrote", out, tokens[:16].tolist())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=0)
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    for name in FIXTURES:
        if a.only and name != a.only:
            continue
        make(name, a.threads)


if __name__ == "__main__":
    main()
