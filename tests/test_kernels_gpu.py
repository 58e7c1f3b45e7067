"""Parity of the sm_100a kernels with the oracle and the reference, through
the C ABI (include/aaedn_b200.h).

Bars: dequant is bit-exact (integer and byte work); the fp32 kernels agree
with the oracle within a bound proportional to the magnitude of the summed
terms: |gpu - oracle| <= 2e-5 * sum_k |x_k * w_k| + 1e-6 (both sides round in
fp32, in a different order, and the GEMV carries x as bf16 hi + lo parts,
2^-18 relative)."""
import numpy as np
import pytest

import aaedn_b200 as ab
from gpu_util import dev, empty_f32, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["d4096", "d1000", "d77", "zero0"])
def test_dequant_bit_exact_vs_reference(ref_golden, name):
    g = ref_golden
    data, scales, want = g[f"dq_{name}_data"], g[f"dq_{name}_scales"], g[f"dq_{name}_out"]
    out = empty_f32(want.size)
    ab.dequant_4bit(dev(data), dev(scales), out, want.size, ab.SCALE_U16INT)
    np.testing.assert_array_equal(host(out).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("n", [1, 31, 32, 33, 4096, 1000003])
def test_dequant_f16_bit_exact_vs_oracle(oracle, n):
    x = ab.synth_normal(5, n, n)
    data, scales = ab.quantize_q4(x)
    out = empty_f32(n)
    ab.dequant_4bit(dev(data), dev(scales), out, n, ab.SCALE_F16)
    want = oracle.dequant(data, scales, n, f16=True)
    np.testing.assert_array_equal(host(out).view(np.uint32), want.view(np.uint32))


def test_dequant_null_inputs_give_zeros():
    out = empty_f32(100)
    ab.dequant_4bit(None, None, out, 100)
    assert np.all(host(out) == 0)


def _q4_matrix(N, K, seed):
    x = ab.synth_normal(seed, 99, N * K)
    return ab.quantize_q4(x)


def _bound(xm, data, scales, N, K, scale_kind, oracle):
    """2e-5 * sum_k |x_k w_k| + 1e-6 per output, from the dequantized matrix."""
    w = oracle.dequant(data, scales, N * K, f16=(scale_kind == ab.SCALE_F16)).reshape(N, K)
    return 2e-5 * (np.abs(xm) @ np.abs(w).T) + 1e-6


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (1, 11008, 4096), (1, 4096, 11008), (8, 4096, 4096),
                                   (8, 11008, 4096), (8, 4096, 11008), (3, 288, 288), (2, 100, 96),
                                   (1, 17, 32), (5, 864, 768), (64, 512, 1024)])
def test_fused_matmul_vs_oracle(oracle, M, N, K):
    data, scales = _q4_matrix(N, K, N + K)
    xm = ab.synth_normal(11, M, M * K, std=1.0).reshape(M, K)
    out = empty_f32(M * N)
    ab.fused_matmul(dev(xm), dev(data), dev(scales), out, M, N, K)
    got = host(out).reshape(M, N)
    want = oracle.q4_matmul(xm, data, scales, N, K)
    err = np.abs(got - want)
    bound = _bound(xm, data, scales, N, K, ab.SCALE_F16, oracle)
    assert np.all(err <= bound), (err.max(), (err / bound).max())


def test_fused_matmul_strides_and_integer_scales(oracle):
    M, N, K, ldb, lda, ldc = 3, 200, 256, 320, 300, 210
    x = ab.synth_normal(3, 1, N * ldb)
    data, _ = ab.quantize_q4(x)
    scales = np.random.default_rng(0).integers(0, 9, N * ldb // 32).astype(np.uint16)
    xm = ab.synth_normal(4, 1, M * lda, std=1.0).reshape(M, lda)
    out = empty_f32(M * ldc)
    ab.fused_matmul(dev(xm), dev(data), dev(scales), out, M, N, K, lda=lda, ldb=ldb, ldc=ldc,
                    scale_kind=ab.SCALE_U16INT)
    got = host(out).reshape(M, ldc)[:, :N]
    want = np.empty((M, N), np.float32)
    import pyoracle
    oracle.lib.or_q4_matmul(pyoracle.ptr(np.ascontiguousarray(xm)), pyoracle.ptr(data), pyoracle.ptr(scales),
                            pyoracle.ptr(want), M, N, K, lda, ldb, N, 1)
    codes = np.stack([data & 15, data >> 4], 1).reshape(N, ldb).astype(np.float32)
    w = (codes * np.repeat(scales.reshape(N, ldb // 32).astype(np.float32), 32, axis=1))[:, :K]
    bound = 2e-5 * (np.abs(xm[:, :K]) @ np.abs(w).T) + 1e-6
    assert np.all(np.abs(got - want) <= bound)


def test_fused_matmul_rejects_bad_shapes():
    out = empty_f32(16)
    with pytest.raises(ab.AaednError):
        ab.fused_matmul(out, out, out, out, 1, 4, 33)  # K not a multiple of 32
    ab.fused_matmul(out, out, out, out, 0, 4, 32)  # M == 0 is a no-op (src/fused_matmul.cpp:76)


def test_f32_matmul_vs_oracle(oracle):
    M, N, K = 2, 1000, 288
    w = ab.synth_normal(8, 0, N * K).reshape(N, K)
    x = ab.synth_normal(8, 1, M * K, std=1.0).reshape(M, K)
    out = empty_f32(M * N)
    ab.f32_matmul(dev(x), dev(w), out, M, N, K)
    want = oracle.f32_matmul(x, w)
    bound = 2e-6 * (np.abs(x) @ np.abs(w).T) + 1e-7
    assert np.all(np.abs(host(out).reshape(M, N) - want) <= bound)


@pytest.mark.parametrize("n", [288, 4096, 19])
def test_rmsnorm_vs_reference(ref_golden, n):
    g = ref_golden
    out = empty_f32(n)
    ab.rmsnorm(dev(g[f"rms_{n}_x"]), out, dev(g[f"rms_{n}_w"]), n)
    np.testing.assert_allclose(host(out), g[f"rms_{n}_out"], rtol=3e-6, atol=1e-7)


@pytest.mark.parametrize("hd", [48, 128])
def test_rope_apply_vs_reference(ref_golden, hd):
    g = ref_golden
    q, k = dev(g[f"rope_{hd}_q_in"]), dev(g[f"rope_{hd}_k_in"])
    ab.rope_apply(q, k, 7, hd, dev(g[f"rope_{hd}_cos"]), dev(g[f"rope_{hd}_sin"]))
    np.testing.assert_allclose(host(q), g[f"rope_{hd}_q_out"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(host(k), g[f"rope_{hd}_k_out"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("hd", [48, 128])
def test_attention_one_head_vs_reference(ref_golden, hd):
    g = ref_golden
    out = empty_f32(hd)
    ab.attention(dev(g[f"attn_{hd}_q"]), dev(g[f"attn_{hd}_k"]), dev(g[f"attn_{hd}_v"]), g[f"attn_{hd}_segs"], out,
                 1, hd, 1.0 / np.sqrt(hd))
    np.testing.assert_allclose(host(out), g[f"attn_{hd}_out"], rtol=2e-5, atol=2e-6)


@pytest.mark.parametrize("H,hd,T", [(4, 128, 1000), (6, 48, 37), (32, 128, 640), (2, 64, 5000)])
def test_attention_multi_head_segments_vs_oracle(oracle, H, hd, T):
    rng = np.random.default_rng(H * T)
    q = rng.normal(0, 1, H * hd).astype(np.float32)
    kc = rng.normal(0, 1, T * H * hd).astype(np.float32)
    vc = rng.normal(0, 1, T * H * hd).astype(np.float32)
    cut = [0, T // 5, T // 2, T]
    segs = np.array([[cut[1], cut[2] - cut[1]], [0, cut[1]], [cut[2], T - cut[2]]], np.uint32)
    out = empty_f32(H * hd)
    scale = 1.0 / np.sqrt(hd)
    ab.attention(dev(q), dev(kc), dev(vc), segs, out, H, hd, scale)
    want = oracle.attention(q, kc, vc, segs, H, hd, scale)
    np.testing.assert_allclose(host(out), want, rtol=2e-5, atol=2e-6)


def test_attention_empty_segments_give_zeros():
    out = empty_f32(128)
    q = dev(np.ones(128, np.float32))
    ab.attention(q, q, q, np.zeros((1, 2), np.uint32), out, 1, 128, 0.1)
    assert np.all(host(out) == 0)


def test_ffn_swiglu_reference_semantics_vs_reference(ref_golden):
    """src/ffn.cpp compiled from the reference sources produced ffn_out."""
    g = ref_golden
    B, Hd, F = (int(v) for v in g["ffn_dims"])
    out = empty_f32(B * Hd)
    ab.ffn_swiglu(dev(g["ffn_x"]), out, B, Hd, F, *(dev(g[f"ffn_{k}"]) for k in ("g", "u", "d", "gs", "us", "ds")),
                  semantics=ab.FFN_REFERENCE)
    np.testing.assert_allclose(host(out), g["ffn_out"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("B,Hd,F", [(1, 4096, 11008), (3, 256, 768)])
def test_ffn_swiglu_model_semantics(B, Hd, F):
    """silu(g) * u with fp16 block scales (the model path's FFN), against an
    fp64 evaluation; bound as for the GEMV."""
    rng = np.random.default_rng(F)
    wg, wu, wd = (ab.quantize_q4(rng.normal(0, 0.02, n).astype(np.float32)) for n in (F * Hd, F * Hd, Hd * F))
    x = rng.normal(0, 1, B * Hd).astype(np.float32)
    out = empty_f32(B * Hd)
    ab.ffn_swiglu(dev(x), out, B, Hd, F, dev(wg[0]), dev(wu[0]), dev(wd[0]), dev(wg[1]), dev(wu[1]), dev(wd[1]),
                  semantics=ab.FFN_MODEL)

    def deq(q, n, k):
        d, s = q
        c = np.stack([d & 15, d >> 4], 1).reshape(-1).astype(np.float64)
        return (c * np.repeat(s.view(np.float16).astype(np.float64), 32)).reshape(n, k)

    G, U, D = deq(wg, F, Hd), deq(wu, F, Hd), deq(wd, Hd, F)
    X = x.reshape(B, Hd).astype(np.float64)
    g, u = X @ G.T, X @ U.T
    act = g / (1 + np.exp(-g)) * u
    want = act @ D.T
    mag = np.abs(act) @ np.abs(D.T)
    err = np.abs(host(out).reshape(B, Hd) - want)
    assert np.all(err <= 1e-4 * mag + 1e-5), float((err / (mag + 1e-9)).max())


def test_ffn_swiglu_null_weights_give_zeros():
    out = empty_f32(2 * 64)
    x = dev(np.ones(2 * 64, np.float32))
    ab.ffn_swiglu(x, out, 2, 64, 96, None, None, None, None, None, None)
    assert np.all(host(out) == 0)
