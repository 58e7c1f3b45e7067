"""Pins the oracle (CPU restatement) to the reference.

* the quantizer must equal the reference's own Python function
  (tools/convert_model.py:36-55) byte for byte on every golden case;
* dequant_4bit must equal the reference C++ (src/dequant.cpp:7-28, compiled
  from source) bit for bit;
* rmsnorm, rope and single-head attention agree with the compiled reference
  to fp32 rounding (the reference is built with -ffast-math);
* the .abn v2 accept/reject decisions match src/quant.cpp:31-119 on the
  fixtures of the reference's own failure-mode tests.
"""
import numpy as np
import pytest


def test_quantizer_bit_exact(oracle, quant_golden):
    g = quant_golden
    for name in g["names"]:
        x = g[f"{name}__x"]
        data, scales = oracle.quantize(x)
        np.testing.assert_array_equal(data, g[f"{name}__data"], err_msg=f"codes {name}")
        np.testing.assert_array_equal(scales, g[f"{name}__scales"], err_msg=f"scales {name}")


def test_fnv1a(oracle, quant_golden):
    assert oracle.fnv1a32(quant_golden["fnv_payload"].tobytes()) == int(quant_golden["fnv_value"][0])


def test_f16_roundtrip_matches_numpy(oracle):
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.normal(0, 1, 2000) * 10.0 ** rng.integers(-9, 6, 2000),
                           [0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 2.0 ** -25, 2.0 ** -24 * 1.5]])
    for v in vals:
        with np.errstate(over="ignore"):  # values past the fp16 range round to inf on purpose
            want = np.array([v]).astype(np.float16).view(np.uint16)[0]
        assert oracle.lib.or_f64_to_f16(float(v)) == want, v
    for h in range(0, 65536, 7):
        f = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        got = oracle.lib.or_f16_to_f32(h)
        if np.isnan(f):
            assert np.isnan(got)
        else:
            assert got == f, h


@pytest.mark.parametrize("name", ["d4096", "d1000", "d77", "zero0"])
def test_dequant_matches_reference(oracle, ref_golden, name):
    g = ref_golden
    data, scales, want = g[f"dq_{name}_data"], g[f"dq_{name}_scales"], g[f"dq_{name}_out"]
    got = oracle.dequant(data, scales, want.size)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("n", [288, 4096, 19])
def test_rmsnorm_matches_reference(oracle, ref_golden, n):
    g = ref_golden
    got = oracle.rmsnorm(g[f"rms_{n}_x"], g[f"rms_{n}_w"])
    np.testing.assert_allclose(got, g[f"rms_{n}_out"], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("hd,ms", [(48, 64), (128, 32)])
def test_rope_matches_reference(oracle, ref_golden, hd, ms):
    """src/rope.cpp:8-34 evaluates pos * 10000/2^(i/half) in fp32; angles reach
    1e5 rad, where the table depends on how powf/cosf are evaluated. Built with
    the reference's own flags (-O3 -mavx2 -mfma -ffast-math: vectorised libm),
    the oracle's restatement reproduces the reference table bit for bit; the
    strict build (scalar libm) is what the CUDA library's table follows."""
    import pyoracle
    g = ref_golden
    fast = pyoracle.Oracle(fast=True)
    c, s = fast.rope_tables_ref(ms, hd)
    np.testing.assert_array_equal(c, g[f"rope_{hd}_cos"])
    np.testing.assert_array_equal(s, g[f"rope_{hd}_sin"])
    # strict build: identical wherever the fp32 angle is small
    c2, s2 = oracle.rope_tables_ref(ms, hd)
    small = (np.arange(ms)[:, None] * 10000.0 / 2 ** (np.arange(hd // 2)[None, :] / (hd // 2))).reshape(-1) < 1.0
    np.testing.assert_allclose(c2[small], c[small], atol=1e-6)
    np.testing.assert_allclose(s2[small], s[small], atol=1e-6)
    q, k = oracle.rope_apply(g[f"rope_{hd}_q_in"], g[f"rope_{hd}_k_in"], 7, hd, g[f"rope_{hd}_cos"],
                             g[f"rope_{hd}_sin"])
    np.testing.assert_allclose(q, g[f"rope_{hd}_q_out"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(k, g[f"rope_{hd}_k_out"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("hd", [48, 128])
def test_attention_one_head_matches_reference(oracle, ref_golden, hd):
    g = ref_golden
    got = oracle.attention(g[f"attn_{hd}_q"], g[f"attn_{hd}_k"], g[f"attn_{hd}_v"], g[f"attn_{hd}_segs"], 1,
                           hd, 1.0 / np.sqrt(hd))
    np.testing.assert_allclose(got, g[f"attn_{hd}_out"], rtol=1e-5, atol=1e-6)


def test_ffn_refsem_matches_reference(oracle, ref_golden):
    import pyoracle
    g = ref_golden
    B, Hd, F = (int(v) for v in g["ffn_dims"])
    out = np.empty(B * Hd, np.float32)
    oracle.lib.or_ffn_swiglu_refsem(*(pyoracle.ptr(a) for a in (g["ffn_x"], out)), B, Hd, F,
                                    *(pyoracle.ptr(g[f"ffn_{k}"]) for k in ("g", "u", "d", "gs", "us", "ds")))
    np.testing.assert_allclose(out, g["ffn_out"], rtol=1e-4, atol=1e-4)


def test_abn_v2_decisions_match_reference(oracle, ref_golden):
    g = ref_golden
    for nm in g["ql_names"]:
        blob = g[f"ql_{nm}_file"].tobytes()
        ok = int(g[f"ql_{nm}_result"][0])
        assert oracle.abn_v2_accepts(blob) == bool(ok), nm
    # the reference rejects its own (mis-sized) roundtrip fixture
    assert int(g["ql_roundtrip_fixture_result"][0]) == 0
    assert int(g["ql_valid_h64_result"][0]) == 1
