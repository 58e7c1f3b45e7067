"""CPU checks of the product's host side: the C ABI library loads and
exports every symbol of include/aaedn_b200.h, and the host quant tools
(block quantizer, FNV-1a, RoPE tables) are bit-exact against the reference
quantizer's golden vectors and the oracle. No kernel is launched."""
import ctypes
import subprocess

import numpy as np
import pytest

import aaedn_b200 as ab


def test_library_exports_every_declared_symbol():
    L = ab.lib()
    names = ab.exported_symbols()
    assert len(names) > 30
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", ab.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if ln.strip()}
    assert set(names) <= exported


def test_version_and_error_state():
    assert ab.lib().aaedn_version() >= 1
    # host-only call with a bad argument sets the thread's last error
    rc = ab.lib().aaedn_synth_tokens(1, 0, 0, None, 4)
    assert rc == ab.EINVAL
    assert "synth_tokens" in ab.last_error()


def test_quantizer_matches_reference_golden(quant_golden):
    g = quant_golden
    for name in g["names"]:
        data, scales = ab.quantize_q4(g[f"{name}__x"])
        np.testing.assert_array_equal(data, g[f"{name}__data"], err_msg=name)
        np.testing.assert_array_equal(scales, g[f"{name}__scales"], err_msg=name)


def test_quantizer_matches_oracle_on_large_input(oracle):
    x = ab.synth_normal(7, 3, 1 << 20)
    d1, s1 = ab.quantize_q4(x)
    d2, s2 = oracle.quantize(x)
    np.testing.assert_array_equal(d1, d2)
    np.testing.assert_array_equal(s1, s2)
    # unsigned quantizer: negative weights become code 0, codes <= 7 in practice
    codes = np.stack([d1 & 15, d1 >> 4], 1).reshape(-1)
    assert codes.max() <= 8 and (codes == 0).mean() > 0.5


def test_fnv1a(quant_golden):
    assert ab.fnv1a32(quant_golden["fnv_payload"].tobytes()) == int(quant_golden["fnv_value"][0])


def test_rope_tables_match_oracle(oracle):
    for hd, ms in ((48, 256), (128, 512)):
        c, s = ab.rope_table(ms, hd, formula=0)
        c2, s2 = oracle.rope_tables_ref(ms, hd)
        np.testing.assert_array_equal(c, c2)
        np.testing.assert_array_equal(s, s2)
        for theta in (10000.0, 500000.0):
            c, s = ab.rope_table(ms, hd, theta, formula=1)
            c2, s2 = oracle.rope_tables(ms, hd, theta)
            np.testing.assert_array_equal(c, c2)
            np.testing.assert_array_equal(s, s2)


def test_synthetic_generator_is_deterministic_and_normal():
    a = ab.synth_normal(1234, 16, 1 << 18)
    b = ab.synth_normal(1234, 16, 1 << 18)
    c = ab.synth_normal(1234, 17, 1 << 18)
    np.testing.assert_array_equal(a, b)
    assert not np.array_equal(a, c)
    assert abs(a.mean()) < 2e-4 and abs(a.std() - 0.02) < 2e-4
    t = ab.synth_tokens(1234, 0, 32000, 10000)
    assert t.max() < 32000 and len(np.unique(t)) > 8000


def _abn(hidden=64, version=2, magic=b"AAEDNMDL", corrupt=False, truncate=0, size_delta=0):
    import struct
    rng = np.random.default_rng(hidden)
    codes = rng.integers(0, 256, hidden * hidden // 2, dtype=np.uint8)
    scales = rng.integers(0, 65536, hidden * hidden // 32, dtype=np.uint16)
    payload = codes.tobytes() + scales.tobytes()
    head = struct.pack("<8sIQI6IB15s", magic, version, len(payload) + size_delta, ab.fnv1a32(payload), 2, 4, 16,
                       1000, hidden, 4 * hidden, 0, b"\x00" * 15)
    blob = bytearray(head + payload)
    if corrupt:
        blob[64 + 5] ^= 1
    if truncate:
        blob = blob[:-truncate]
    return bytes(blob), codes, scales


@pytest.mark.parametrize("case", ["valid", "magic", "version", "size", "checksum", "short", "header"])
def test_abn_reader_matches_oracle(oracle, tmp_path, case):
    """quant_load's checks (src/quant.cpp:50-111) in the host reader, and the
    oracle's restatement of them, give the same decision."""
    kw = {"valid": {}, "magic": {"magic": b"AAEDNXXX"}, "version": {"version": 3}, "size": {"size_delta": 2},
          "checksum": {"corrupt": True}, "short": {"truncate": 3}, "header": {"truncate": 10 ** 6}}[case]
    blob, codes, scales = _abn(**kw) if case != "header" else (_abn()[0][:40], None, None)
    path = tmp_path / f"{case}.abn"
    path.write_bytes(blob)
    accepted = oracle.abn_v2_accepts(blob)
    try:
        h, data, sc = ab.abn_read(path)
        ok = True
    except ab.AaednError as e:
        assert e.rc == ab.EFORMAT
        ok = False
    assert ok == accepted == (case == "valid")
    if ok:
        assert h.version == 2 and h.hidden_dim == 64 and h.vocab_size == 1000
        np.testing.assert_array_equal(data, codes)
        np.testing.assert_array_equal(sc, scales)


WHOLE = dict(dim=256, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=32, ffn_dim=512, vocab=1000, max_seq=200,
             rope_theta=500000.0, eps=1e-6)


def test_whole_model_file_header_round_trip(tmp_path):
    import abn_model_file
    w = ab.synthetic_weights(WHOLE, 31)
    path = tmp_path / "m.abn"
    n = abn_model_file.write(path, WHOLE, w)
    cfg = ab.abn_model_config(path, max_seq=200)
    assert cfg == {**WHOLE, "rope_theta": np.float32(WHOLE["rope_theta"]), "eps": np.float32(WHOLE["eps"])}
    assert path.stat().st_size == 64 + n


def test_whole_model_file_rejections(tmp_path):
    import abn_model_file
    w = ab.synthetic_weights(WHOLE, 31)
    good = tmp_path / "good.abn"
    abn_model_file.write(good, WHOLE, w)
    raw = good.read_bytes()
    cases = {
        "short": raw[:40],
        "magic": b"X" + raw[1:],
        "v2": raw[:8] + (2).to_bytes(4, "little") + raw[12:],               # a one-matrix file's version
        "size": raw[:12] + (len(raw) - 65).to_bytes(8, "little") + raw[20:],  # payload_size off by one
        "kv": raw[:49] + (3).to_bytes(4, "little") + raw[53:],               # 8 heads over 3 kv heads
    }
    for name, blob in cases.items():
        p = tmp_path / f"{name}.abn"
        p.write_bytes(blob)
        with pytest.raises(ab.AaednError) as e:
            ab.abn_model_config(p)
        assert e.value.rc == ab.EFORMAT, name
    # the one-matrix reader keeps rejecting whole-model files (version 3)
    with pytest.raises(ab.AaednError):
        ab.abn_read(good)


def test_oracle_generator_matches_the_library(oracle):
    """The oracle's restatement of the seeded generator (what bench.py's CPU
    arm and the fixture script build their weights from) gives the library's
    synthetic tensors and prompts bit for bit, and its quantizer the
    library's codes and scales."""
    import pyoracle
    for seed, tid, n in ((1234, 0, 1001), (7, 16 + 8 * 3 + 6, 300001), (1, 1, 5)):
        a = ab.synth_normal(seed, tid, n)
        b = oracle.synth_normal(seed, tid, n)
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    np.testing.assert_array_equal(ab.synth_tokens(1234, 0, 32000, 128), oracle.synth_tokens(1234, 0, 32000, 128))
    cfg = dict(ab.TINY, n_layers=2)
    w1, w2 = ab.synthetic_weights(cfg, 1234), pyoracle.synthetic_weights(cfg, 1234, oracle)
    for k in ab.LAYER_MATS:
        for l in range(2):
            for i in range(2):
                np.testing.assert_array_equal(w1[k][l][i], w2[k][l][i])
    np.testing.assert_array_equal(w1["embedding"], w2["embedding"])
    np.testing.assert_array_equal(w1["lm_head"], w2["lm_head"])


def test_oracle_seek_fills_the_cache_below_the_position(oracle):
    """The CPU baseline's timing aid: after seek(p) the next step runs at
    position p (its logits are finite; attention reads p + 1 rows)."""
    import pyoracle
    cfg = dict(ab.TINY, n_layers=1, max_seq=64)
    om = pyoracle.OracleModel(oracle, cfg, pyoracle.synthetic_weights(cfg, 3, oracle))
    om.seek(40)
    assert om.pos == 40
    lg = om.step(5)
    assert om.pos == 41 and np.isfinite(lg).all()
    with pytest.raises(ValueError):
        om.seek(64)
