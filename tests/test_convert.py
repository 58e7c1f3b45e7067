"""The whole-model .abn writer (aaedn_abn_model_write) and the checkpoint
converter (python -m aaedn_b200.convert), on the CPU.

The writer's file is byte-identical to the independent test writer
(tests/abn_model_file.py, which follows the documented layout field by
field), its header reads back as the model's shape, and a Llama-style
safetensors checkpoint converts into the same bytes as its tensors
quantized with the block quantizer (tools/convert_model.py:36-55) and
written directly."""
import json
import struct

import numpy as np

import aaedn_b200 as ab
from aaedn_b200 import convert
import abn_model_file

GQA = dict(dim=256, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=32, ffn_dim=512, vocab=300, max_seq=64,
           rope_theta=500000.0, eps=1e-5)


def _same_shape(got, want):
    # the header keeps theta and eps as fp32
    assert {k: v for k, v in got.items() if k not in ("rope_theta", "eps")} == \
        {k: v for k, v in want.items() if k not in ("rope_theta", "eps")}
    assert got["rope_theta"] == np.float32(want["rope_theta"]) and got["eps"] == np.float32(want["eps"])


def test_writer_matches_the_documented_layout(tmp_path):
    w = ab.synthetic_weights(GQA, 3)
    a, b = tmp_path / "a.abn", tmp_path / "b.abn"
    convert.write_abn_model(a, GQA, w)
    abn_model_file.write(b, GQA, w)
    assert a.read_bytes() == b.read_bytes()
    _same_shape(ab.abn_model_config(a, max_seq=GQA["max_seq"]), GQA)


def _write_safetensors(path, tensors):
    hdr, off, blobs = {}, 0, []
    for name, arr in tensors.items():
        raw = np.ascontiguousarray(arr).tobytes()
        dt = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16"}[arr.dtype]
        hdr[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def test_safetensors_checkpoint_converts(tmp_path):
    cfg = GQA
    rng = np.random.default_rng(0)
    D, F, V, hd = cfg["dim"], cfg["ffn_dim"], cfg["vocab"], cfg["head_dim"]
    qd, kd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    t = {"model.embed_tokens.weight": rng.normal(0, 0.02, (V, D)).astype(np.float32),
         "model.norm.weight": rng.uniform(0.5, 1.5, D).astype(np.float32),
         "lm_head.weight": rng.normal(0, 0.02, (V, D)).astype(np.float16)}
    shapes = {"self_attn.q_proj": (qd, D), "self_attn.k_proj": (kd, D), "self_attn.v_proj": (kd, D),
              "self_attn.o_proj": (D, qd), "mlp.gate_proj": (F, D), "mlp.up_proj": (F, D), "mlp.down_proj": (D, F)}
    for l in range(cfg["n_layers"]):
        for n, s in shapes.items():
            t[f"model.layers.{l}.{n}.weight"] = rng.normal(0, 0.02, s).astype(np.float32)
        t[f"model.layers.{l}.input_layernorm.weight"] = rng.uniform(0.5, 1.5, D).astype(np.float32)
        t[f"model.layers.{l}.post_attention_layernorm.weight"] = rng.uniform(0.5, 1.5, D).astype(np.float32)
    st = tmp_path / "m.safetensors"
    _write_safetensors(st, t)
    hc = tmp_path / "config.json"
    hc.write_text(json.dumps({"num_attention_heads": 8, "num_key_value_heads": 2, "rope_theta": 500000.0,
                              "rms_norm_eps": 1e-5}))
    out = tmp_path / "m.abn"
    convert.main(["--model", str(st), "--config", str(hc), "--output", str(out)])
    # the same tensors quantized and written directly
    names = dict(zip(ab.LAYER_MATS, shapes))
    w = {k: [ab.quantize_q4(t[f"model.layers.{l}.{names[k]}.weight"]) for l in range(2)] for k in ab.LAYER_MATS}
    w["attn_norm"] = [t[f"model.layers.{l}.input_layernorm.weight"] for l in range(2)]
    w["ffn_norm"] = [t[f"model.layers.{l}.post_attention_layernorm.weight"] for l in range(2)]
    w["embedding"] = t["model.embed_tokens.weight"]
    w["lm_head"] = t["lm_head.weight"].astype(np.float32)
    w["final_norm"] = t["model.norm.weight"]
    ref = tmp_path / "ref.abn"
    abn_model_file.write(ref, dict(cfg, max_seq=0), w)
    assert out.read_bytes() == ref.read_bytes()
    _same_shape(ab.abn_model_config(out, max_seq=64), cfg)
