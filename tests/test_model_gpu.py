"""End-to-end parity of the decode loop with the oracle (CPU restatement of
src/transformer.cpp:128-243 with the documented decisions), through the
C ABI.

Bars (from the task's correctness definition): identical greedy tokens
(the tiny config: all 248 decode steps; the first 64 at least on every
config), logits within max-abs <= 1e-2 * max|logit| (checked much tighter
here: 1e-4), per-layer hidden states within 1e-4 relative."""
import numpy as np
import pytest

import aaedn_b200 as ab
import pyoracle

pytestmark = pytest.mark.gpu

SEED = 1234
GQA_SMALL = dict(dim=256, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=32, ffn_dim=512, vocab=1000, max_seq=200,
                 rope_theta=500000.0, eps=1e-6)


def _pair(cfg, seed=SEED):
    w = ab.synthetic_weights(cfg, seed)
    om = pyoracle.OracleModel(pyoracle.Oracle(), cfg, w)
    gm = ab.Model(cfg)
    gm.set_weights(w)
    return w, om, gm


@pytest.fixture(scope="module")
def tiny():
    w, om, gm = _pair(ab.TINY)
    yield ab.TINY, w, om, gm
    gm.close()


def _rel_err(a, b):
    return float(np.abs(a - b).max() / max(1e-30, np.abs(b).max()))


def test_tiny_greedy_248_tokens_identical(tiny):
    cfg, w, om, gm = tiny
    prompt = ab.synth_tokens(SEED, 0, cfg["vocab"], 8)
    om.reset()
    gm.reset()
    want, want_logits = om.generate(prompt, 248)
    got = gm.generate(prompt, 248)
    first = np.nonzero(got != want)[0]
    assert first.size == 0, f"first mismatch at step {first[0]}"
    assert gm.pos == om.pos == 8 + 247
    assert _rel_err(gm.logits(), want_logits) < 1e-4


def test_tiny_forward_logits_and_hidden(tiny):
    cfg, w, om, gm = tiny
    prompt = ab.synth_tokens(SEED, 1, cfg["vocab"], 12)
    om.reset()
    gm.reset()
    for t in prompt[:-1]:
        om.step(t)
    lg = gm.forward(prompt[:-1])
    want_logits, want_hidden = om.step(prompt[-1], want_hidden=True)
    hid, got_logits = gm.forward_debug(prompt[-1])
    for l in range(cfg["n_layers"]):
        assert _rel_err(hid[l], want_hidden[l]) < 1e-4, l
    assert _rel_err(got_logits, want_logits) < 1e-4
    assert np.argmax(got_logits) == np.argmax(want_logits)
    assert lg is not None and np.isfinite(lg).all()


def test_decode_steps_continue_generate(tiny):
    cfg, w, om, gm = tiny
    prompt = ab.synth_tokens(SEED, 2, cfg["vocab"], 5)
    gm.reset()
    ref = gm.generate(prompt, 40)
    gm.reset()
    first = gm.generate(prompt, 10)
    gm.decode_steps(30)
    np.testing.assert_array_equal(first, ref[:10])
    np.testing.assert_array_equal(gm.tokens(40), ref)


def test_synthesize_equals_python_weights(tiny):
    cfg, w, om, gm = tiny
    prompt = ab.synth_tokens(SEED, 3, cfg["vocab"], 6)
    gm.reset()
    a = gm.forward(prompt)
    with ab.Model(cfg) as g2:
        g2.synthesize(SEED)
        b = g2.forward(prompt)
    np.testing.assert_array_equal(a, b)


def test_sequence_bounds_and_bad_tokens(tiny):
    cfg, w, om, gm = tiny
    gm.reset()
    with pytest.raises(ab.AaednError):
        gm.forward(np.array([cfg["vocab"]], np.uint32))
    with pytest.raises(ab.AaednError):
        gm.forward(np.zeros(cfg["max_seq"] + 1, np.uint32))
    gm.reset()
    with pytest.raises(ab.AaednError):
        gm.decode_steps(1)  # nothing in the sequence yet


def test_gqa_greedy_identical():
    cfg = GQA_SMALL
    w, om, gm = _pair(cfg, seed=77)
    prompt = ab.synth_tokens(77, 0, cfg["vocab"], 9)
    want, wl = om.generate(prompt, 120)
    got = gm.generate(prompt, 120)
    np.testing.assert_array_equal(got, want)
    assert _rel_err(gm.logits(), wl) < 1e-4
    gm.close()


def test_7b_width_two_layers_vs_oracle():
    """Full 7B widths (dim 4096, 32 heads x 128, ffn 11008, vocab 32000): the
    full-size GEMV/attention shapes, two layers so the oracle stays fast."""
    cfg = dict(ab.LLAMA2_7B, n_layers=2, max_seq=256)
    w, om, gm = _pair(cfg, seed=2024)
    prompt = ab.synth_tokens(2024, 0, cfg["vocab"], 4)
    want, wl = om.generate(prompt, 64)
    got = gm.generate(prompt, 64)
    np.testing.assert_array_equal(got, want)
    assert _rel_err(gm.logits(), wl) < 1e-4
    gm.close()


@pytest.mark.parametrize("env", [
    {"AAEDN_ATTN_CLUSTER": "0", "AAEDN_ATTN_CTAS_PER_SM": "4"},  # splits merged in global memory, S > 16
    {"AAEDN_ATTN_CLUSTER": "16"},             # clusters of 16 splits (non-portable size)
    {"AAEDN_PDL": "0", "AAEDN_L2HINT": "0"},  # plain launches, no L2 policy
    {"AAEDN_GEMV_STAGES": "12"},              # the deepest ring of the decode GEMV
    {"AAEDN_GEMV_STAGES": "4"},               # the shallowest
    {"AAEDN_ATTN_WARPS": "8"},                # decode attention CTAs of 8 warps
    {"AAEDN_ATTN_WARPS": "10"},               # of 10 warps
])
def test_launch_options_same_tokens(env, monkeypatch):
    """The model's launch options (read when it is created) change timing
    only: the 7B widths, two layers, against the oracle."""
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    cfg = dict(ab.LLAMA2_7B, n_layers=2, max_seq=256)
    w, om, gm = _pair(cfg, seed=99)
    prompt = ab.synth_tokens(99, 0, cfg["vocab"], 5)
    want, wl = om.generate(prompt, 48)
    got = gm.generate(prompt, 48)
    np.testing.assert_array_equal(got, want)
    assert _rel_err(gm.logits(), wl) < 1e-4
    gm.close()


def test_launch_count_per_step():
    """Every kernel of the decode step is counted (the bench reports the
    count): 5 per layer (qkv, attention, o, gate/up, down) and the lm_head."""
    cfg = GQA_SMALL
    w, om, gm = _pair(cfg, seed=5)
    gm.forward(ab.synth_tokens(5, 0, cfg["vocab"], 3), want_logits=False)
    assert gm.kernels_per_step == 5 * cfg["n_layers"] + 1
    n0 = ab.kernel_launches()
    gm.decode_steps(2)
    gm.status()
    assert ab.kernel_launches() - n0 == 2 * (5 * cfg["n_layers"] + 1)
    gm.close()


def test_model_from_whole_model_file(tmp_path):
    """aaedn_model_load_abn: a whole-model .abn file gives the same greedy
    tokens and logits as the same weights handed over in memory (the oracle's);
    a corrupted payload or a nonzero QKV bias is refused before any weight of
    the model changes."""
    import abn_model_file
    cfg = GQA_SMALL
    w = ab.synthetic_weights(cfg, 41)
    path = tmp_path / "m.abn"
    abn_model_file.write(path, cfg, w)
    gm = ab.Model(ab.abn_model_config(path, max_seq=cfg["max_seq"]))
    gm.load_abn(path)
    om = pyoracle.OracleModel(pyoracle.Oracle(), cfg, w)
    prompt = ab.synth_tokens(41, 0, cfg["vocab"], 6)
    want, wl = om.generate(prompt, 40)
    np.testing.assert_array_equal(gm.generate(prompt, 40), want)
    assert _rel_err(gm.logits(), wl) < 1e-4
    raw = bytearray(path.read_bytes())
    raw[-1] ^= 1
    bad = tmp_path / "bad.abn"
    bad.write_bytes(bytes(raw))
    with pytest.raises(ab.AaednError) as e:
        gm.load_abn(bad)
    assert e.value.rc == ab.EFORMAT
    biased = tmp_path / "bias.abn"
    abn_model_file.write(biased, cfg, w, bias=np.full((cfg["n_heads"] + 2 * cfg["n_kv_heads"]) * cfg["head_dim"], 0.5))
    with pytest.raises(ab.AaednError) as e:
        gm.load_abn(biased)
    assert e.value.rc == ab.EUNSUPPORTED
    gm.reset()
    np.testing.assert_array_equal(gm.generate(prompt, 40), want)  # the refused files changed nothing
    gm.close()
