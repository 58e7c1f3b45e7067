"""Prefill through the tensor-core GEMM (prompt tokens processed together:
src/transformer.cpp:128-243 with decision D7) against the oracle, which
processes the same prompt one token at a time.

The model takes this path for a multi-token forward / generate when every
matrix has the tile-major layout (K a multiple of 128, N of 16). Checked:
the logits after the prompt, the greedy tokens that follow (decoded by the
per-token graph from the cache the prefill wrote), prompts split into
several chunks, a prompt that continues a sequence already in the cache,
and GQA. Bars as the other model tests: tokens identical, logits within
1e-4 relative max-abs."""
import numpy as np
import pytest

import aaedn_b200 as ab
import pyoracle

pytestmark = pytest.mark.gpu

GQA_SMALL = dict(dim=256, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=32, ffn_dim=512, vocab=1000, max_seq=320,
                 rope_theta=500000.0, eps=1e-6)


def _rel_err(a, b):
    return float(np.abs(a - b).max() / max(1e-30, np.abs(b).max()))


def _pair(cfg, seed):
    w = ab.synthetic_weights(cfg, seed)
    om = pyoracle.OracleModel(pyoracle.Oracle(), cfg, w)
    gm = ab.Model(cfg)
    gm.set_weights(w)
    return w, om, gm


@pytest.mark.parametrize("n_prompt", [2, 37, 128])
def test_prefill_logits_and_tokens_vs_oracle(n_prompt):
    cfg = dict(ab.LLAMA2_7B, n_layers=2, max_seq=256)
    w, om, gm = _pair(cfg, seed=300 + n_prompt)
    prompt = ab.synth_tokens(300 + n_prompt, 0, cfg["vocab"], n_prompt)
    want_lp = None
    for t in prompt:
        want_lp = om.step(int(t))
    lp = gm.forward(prompt)
    assert _rel_err(lp, want_lp) < 1e-4
    om.reset()
    gm.reset()
    want, wl = om.generate(prompt, 32)
    got = gm.generate(prompt, 32)
    np.testing.assert_array_equal(got, want)
    assert _rel_err(gm.logits(), wl) < 1e-4
    gm.close()


def test_prefill_in_chunks_and_continued_sequence(monkeypatch):
    """Chunks of 16 rows (AAEDN_PREFILL_ROWS, read at model creation): a
    70-token prompt takes 5 chunks, each attending to the cache the earlier
    ones wrote; then a second 20-token forward continues the sequence."""
    monkeypatch.setenv("AAEDN_PREFILL_ROWS", "16")
    cfg = GQA_SMALL
    w, om, gm = _pair(cfg, seed=71)
    p1 = ab.synth_tokens(71, 0, cfg["vocab"], 70)
    p2 = ab.synth_tokens(71, 1, cfg["vocab"], 20)
    for t in np.concatenate([p1, p2]):
        want = om.step(int(t))
    gm.forward(p1, want_logits=False)
    got = gm.forward(p2)
    assert gm.pos == 90
    assert _rel_err(got, want) < 1e-4
    # decoding continues from the prefilled cache
    tok = int(np.argmax(want))
    assert gm.next_token() == tok
    nxt = om.step(tok)
    gm.decode_steps(1)
    assert gm.next_token() == int(np.argmax(nxt))
    gm.close()


def test_prefill_gqa_long_prompt_vs_oracle():
    cfg = GQA_SMALL
    w, om, gm = _pair(cfg, seed=9)
    prompt = ab.synth_tokens(9, 0, cfg["vocab"], 300)  # 256-row chunk + 44
    want, wl = om.generate(prompt, 16)
    np.testing.assert_array_equal(gm.generate(prompt, 16), want)
    assert _rel_err(gm.logits(), wl) < 1e-4
    gm.close()
