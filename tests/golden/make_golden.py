#!/usr/bin/env python3
"""Generate the golden fixtures that pin the oracle to the reference.

Run where the reference checkout exists, named by the AAEDN_REF environment
variable (required), with oracle/_ref built from it
(``make -C oracle AAEDN_REF=...``). Writes two small files next to this
script:

* ``quant_golden.npz`` — inputs and outputs of the reference's own block
  quantizer ``quantize_block_4bit_unsigned`` (tools/convert_model.py:36-55),
  imported from the reference checkout, on seeded inputs plus edge cases
  (all-zero and all-negative blocks, ragged tails, rounding ties, fp16
  subnormal and overflowing scales).
* ``ref_kernels_golden.npz`` — outputs of the reference C++ kernels compiled
  from source (oracle/_ref/libaaedn_ref.so): dequant_4bit
  (src/dequant.cpp:7-28), rmsnorm (src/rmsnorm.cpp:8-51), rope_init /
  rope_apply (src/rope.cpp:8-63), attention with one head
  (src/attention.cpp:10-84), ffn_swiglu (src/ffn.cpp:18-77) and the
  accept/reject decisions of quant_load (src/quant.cpp:31-119) on the
  fixtures of tests/test_startup_failure.cpp and
  tests/test_artifact_roundtrip.cpp.

The fixtures are committed; the GPU box never needs the reference checkout.
"""
import ctypes
import importlib.util
import os
import struct
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("AAEDN_REF")  # the reference project's root: required


def load_reference_quantizer():
    path = os.path.join(REF, "tools", "convert_model.py")
    spec = importlib.util.spec_from_file_location("aaedn_ref_convert_model", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def quant_cases(rng):
    cases = []
    # seeded N(0, 0.02) weights, the distribution the synthetic models use
    cases.append(("normal_4096", rng.normal(0.0, 0.02, 4096).astype(np.float32)))
    cases.append(("normal_ragged_1000", rng.normal(0.0, 0.02, 1000).astype(np.float32)))
    cases.append(("unit_normal_odd_77", rng.normal(0.0, 1.0, 77).astype(np.float32)))
    z = np.zeros(96, np.float32)
    z[40:50] = rng.normal(0, 1, 10)
    cases.append(("zero_blocks", z))
    cases.append(("all_negative", -np.abs(rng.normal(0, 0.5, 64)).astype(np.float32)))
    # exact rounding ties: max 7.0 -> scale 1.0, values k + 0.5
    t = np.array([7.0] + [k + 0.5 for k in range(0, 8)] + [0.5, 1.5, 2.5, 3.5] * 5 + [6.5, 7.0, 0.49999997],
                 dtype=np.float32)[:32]
    cases.append(("ties", t))
    cases.append(("tiny_subnormal_scale", (rng.normal(0, 1, 64) * 1e-5).astype(np.float32)))
    cases.append(("huge_overflow_scale", (rng.normal(0, 1, 64) * 1e6).astype(np.float32)))
    cases.append(("uniform_wide", rng.uniform(-3, 3, 512).astype(np.float32)))
    cases.append(("single", np.array([0.25], np.float32)))
    return cases


def make_quant_golden(mod, rng):
    out = {}
    names = []
    for name, x in quant_cases(rng):
        data, scales = mod.quantize_block_4bit_unsigned(x)
        out[f"{name}__x"] = x
        out[f"{name}__data"] = np.frombuffer(data, np.uint8).copy()
        out[f"{name}__scales"] = np.frombuffer(scales, np.uint16).copy()
        names.append(name)
    out["names"] = np.array(names)
    # FNV-1a of a payload, tools/convert_model.py:16-21
    payload = bytes(range(256)) * 3
    out["fnv_payload"] = np.frombuffer(payload, np.uint8).copy()
    out["fnv_value"] = np.array([mod.fnv1a32(payload)], np.uint32)
    return out


def f32p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def load_ref_lib():
    path = os.path.join(REPO, "oracle", "_ref", "libaaedn_ref.so")
    lib = ctypes.CDLL(path)
    sz = ctypes.c_size_t
    vp = ctypes.c_void_p
    lib.ref_dequant_4bit.argtypes = [vp, vp, vp, sz]
    lib.ref_rmsnorm.argtypes = [vp, vp, vp, sz, ctypes.c_float]
    lib.ref_rope_init.argtypes = [vp, vp, sz, sz]
    lib.ref_rope_apply.argtypes = [vp, vp, sz, sz, vp, vp, sz]
    lib.ref_attention.argtypes = [vp, vp, vp, vp, sz, vp, sz, sz, ctypes.c_float]
    lib.ref_ffn_swiglu.argtypes = [vp, vp, sz, sz, sz, vp, vp, vp, vp, vp, vp]
    lib.ref_quant_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64),
                                   ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32)]
    lib.ref_quant_load.restype = ctypes.c_int
    return lib


def abn_v2(hidden, payload, checksum=None, version=2, magic=b"AAEDNMDL"):
    """Header layout of tools/convert_model.py:137-151 ("<8sIQI6IB15s")."""
    if checksum is None:
        h = 0x811C9DC5
        for b in payload:
            h ^= b
            h = (h * 0x01000193) & 0xFFFFFFFF
        checksum = h
    hdr = struct.pack("<8sIQI6IB15s", magic, version, len(payload), checksum, 24, 16, 64, 32768, hidden,
                      16, 0, b"\x00" * 15)
    return hdr + payload


def make_ref_kernels_golden(lib, rng):
    out = {}
    # dequant_4bit: integer-cast scales, ragged n, zero scale[0] rule
    for name, n in (("d4096", 4096), ("d1000", 1000), ("d77", 77)):
        nb = (n + 31) // 32
        data = rng.integers(0, 256, (n + 1) // 2, dtype=np.uint8)
        scales = rng.integers(1, 65536, nb, dtype=np.uint16)
        o = np.empty(n, np.float32)
        lib.ref_dequant_4bit(f32p(data), f32p(scales), f32p(o), n)
        out[f"dq_{name}_data"], out[f"dq_{name}_scales"], out[f"dq_{name}_out"] = data, scales, o
    data = rng.integers(0, 256, 32, dtype=np.uint8)
    scales = np.array([0, 5], np.uint16)
    o = np.full(64, 7.0, np.float32)
    lib.ref_dequant_4bit(f32p(data), f32p(scales), f32p(o), 64)
    out["dq_zero0_data"], out["dq_zero0_scales"], out["dq_zero0_out"] = data, scales, o

    # rmsnorm at the model widths and a ragged width
    for n in (288, 4096, 19):
        x = rng.normal(0, 1, n).astype(np.float32)
        w = rng.normal(1, 0.1, n).astype(np.float32)
        o = np.empty(n, np.float32)
        lib.ref_rmsnorm(f32p(x), f32p(o), f32p(w), n, 1e-6)
        out[f"rms_{n}_x"], out[f"rms_{n}_w"], out[f"rms_{n}_out"] = x, w, o

    # rope_init tables (reference formula) and rope_apply
    for hd, ms in ((48, 64), (128, 32)):
        half = hd // 2
        c = np.empty(ms * half, np.float32)
        s = np.empty(ms * half, np.float32)
        lib.ref_rope_init(f32p(c), f32p(s), ms, hd)
        out[f"rope_{hd}_cos"], out[f"rope_{hd}_sin"] = c, s
        seq = 7
        q = rng.normal(0, 1, seq * hd).astype(np.float32)
        k = rng.normal(0, 1, seq * hd).astype(np.float32)
        out[f"rope_{hd}_q_in"], out[f"rope_{hd}_k_in"] = q.copy(), k.copy()
        lib.ref_rope_apply(f32p(q), f32p(k), seq, hd, f32p(c), f32p(s), ms)
        out[f"rope_{hd}_q_out"], out[f"rope_{hd}_k_out"] = q, k

    # attention with one head (the reference ignores the head index, so only
    # n_heads == 1 is well defined), two segments
    for hd, T in ((48, 40), (128, 100)):
        q = rng.normal(0, 1, hd).astype(np.float32)
        kc = rng.normal(0, 1, T * hd).astype(np.float32)
        vc = rng.normal(0, 1, T * hd).astype(np.float32)
        segs = np.array([0, T // 3, T // 2, T - T // 2], np.uint32)
        o = np.empty(hd, np.float32)
        lib.ref_attention(f32p(q), f32p(kc), f32p(vc), f32p(segs), 2, f32p(o), 1, hd, 1.0 / np.sqrt(hd))
        for nm, a in (("q", q), ("k", kc), ("v", vc), ("segs", segs), ("out", o)):
            out[f"attn_{hd}_{nm}"] = a

    # ffn_swiglu with the reference layout (ffn_dim <= 4096)
    B, Hd, F = 2, 64, 96
    x = rng.normal(0, 1, B * Hd).astype(np.float32)
    g = rng.integers(0, 256, F * Hd // 2, dtype=np.uint8)
    u = rng.integers(0, 256, F * Hd // 2, dtype=np.uint8)
    d = rng.integers(0, 256, Hd * F // 2, dtype=np.uint8)
    gs = rng.integers(0, 3, F, dtype=np.uint16)  # indexed j/32 -> only F/32 used
    us = rng.integers(0, 3, F, dtype=np.uint16)
    ds = rng.integers(0, 3, Hd, dtype=np.uint16)
    # small scales keep g*silu(g)*u finite
    x *= 0.05
    o = np.empty(B * Hd, np.float32)
    lib.ref_ffn_swiglu(f32p(x), f32p(o), B, Hd, F, f32p(g), f32p(u), f32p(d), f32p(gs), f32p(us), f32p(ds))
    for nm, a in (("x", x), ("g", g), ("u", u), ("d", d), ("gs", gs), ("us", us), ("ds", ds), ("out", o)):
        out[f"ffn_{nm}"] = a
    out["ffn_dims"] = np.array([B, Hd, F], np.int64)

    # quant_load decisions (src/quant.cpp:31-119) on the reference tests'
    # fixtures and a valid file
    files = {}
    files["bad_magic"] = bytes([0xAA]) * 64  # tests/test_startup_failure.cpp:20-23
    files["bad_checksum"] = abn_v2(4, bytes([0x11]) * 10, checksum=0xDEADBEEF)  # :25-55
    files["roundtrip_fixture"] = abn_v2(4, bytes([0x12, 0x34, 0x56, 0x78, 0, 0]) + struct.pack("<HH", 1000, 2000))
    h = 64
    payload = rng.integers(0, 256, h * h // 2, dtype=np.uint8).tobytes() + \
        rng.integers(0, 65536, h * h // 32, dtype=np.uint16).tobytes()
    files["valid_h64"] = abn_v2(h, payload)
    files["bad_version"] = abn_v2(h, payload, version=1)
    files["truncated"] = abn_v2(h, payload)[:-5]
    files["short_header"] = abn_v2(h, payload)[:40]
    names = []
    with tempfile.TemporaryDirectory() as td:
        for nm, blob in files.items():
            p = os.path.join(td, nm + ".abn")
            with open(p, "wb") as f:
                f.write(blob)
            nbk, ver, cks = ctypes.c_uint64(), ctypes.c_uint32(), ctypes.c_uint32()
            ok = lib.ref_quant_load(p.encode(), ctypes.byref(nbk), ctypes.byref(ver), ctypes.byref(cks))
            out[f"ql_{nm}_file"] = np.frombuffer(blob, np.uint8).copy()
            out[f"ql_{nm}_result"] = np.array([ok, nbk.value, ver.value, cks.value], np.uint64)
            names.append(nm)
    out["ql_names"] = np.array(names)
    return out


def main():
    if not REF or not os.path.isdir(os.path.join(REF, "src")):
        raise SystemExit("set AAEDN_REF to the reference project's root (the directory holding src/ and tools/)")
    rng = np.random.default_rng(20261201)
    mod = load_reference_quantizer()
    q = make_quant_golden(mod, rng)
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **q)
    lib = load_ref_lib()
    k = make_ref_kernels_golden(lib, rng)
    np.savez_compressed(os.path.join(HERE, "ref_kernels_golden.npz"), **k)
    for fn in ("quant_golden.npz", "ref_kernels_golden.npz"):
        print(fn, os.path.getsize(os.path.join(HERE, fn)), "bytes")


if __name__ == "__main__":
    sys.exit(main())
