"""Whole-model converter: a Llama-style checkpoint (safetensors, Hugging Face
tensor names) into the whole-model .abn file that aaedn_model_load_abn
(transformer_init) reads.

The reference's tools/convert_model.py writes a single hidden x hidden
matrix under the version-2 header (its lines 121-150); this converter writes
every tensor of the model in the per-layer order of docs/mpd.md:497-499
through aaedn_abn_model_write, quantizing the linear weights with the
library's block quantizer (bit-exact with tools/convert_model.py:36-55).

    python -m aaedn_b200.convert --model model.safetensors [--config config.json] --output model.abn

Tensor names: model.embed_tokens.weight, model.layers.<l>.input_layernorm.weight,
.self_attn.{q,k,v,o}_proj.weight, .post_attention_layernorm.weight,
.mlp.{gate,up,down}_proj.weight, model.norm.weight, lm_head.weight (absent:
tied to the embedding). Heads, KV heads, RoPE theta and eps come from the
Hugging Face config.json when given (num_attention_heads,
num_key_value_heads, rope_theta, rms_norm_eps), else head_dim 128 and
theta 10000, eps 1e-6. Weights are [out][in] row-major (decision D2); q and
k rows are used as stored (the rotate-half RoPE of decision D3 is the
Hugging Face convention).
"""
import argparse
import ctypes
import json
import os
import struct

import numpy as np

from . import LAYER_MATS, LayerHost, ModelConfig, _p, check, lib, quantize_q4

_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": "bf16", "F64": np.float64}


def read_safetensors(path):
    """{name: fp32 array} of a .safetensors file (the format: an 8-byte
    little-endian header length, a JSON header of dtype / shape /
    data_offsets per tensor, then the raw data)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
    base = 8 + n
    raw = np.memmap(path, np.uint8, "r")
    out = {}
    for name, meta in hdr.items():
        if name == "__metadata__":
            continue
        dt = _DTYPES.get(meta["dtype"])
        if dt is None:
            raise ValueError(f"{name}: dtype {meta['dtype']} not supported")
        b0, b1 = meta["data_offsets"]
        buf = raw[base + b0:base + b1]
        if dt == "bf16":
            a = (buf.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            a = buf.view(dt).astype(np.float32)
        out[name] = a.reshape(meta["shape"])
    return out


def write_abn_model(path, cfg, w):
    """Writes host weights in the layout of aaedn_b200.synthetic_weights (per
    layer lists of (codes, fp16 scales) and fp32 arrays) as a whole-model
    .abn file."""
    L = cfg["n_layers"]
    c = ModelConfig(**{k: cfg.get(k, 0) for k, _ in ModelConfig._fields_})
    layers = (LayerHost * L)()
    keep = []
    for l in range(L):
        for name in LAYER_MATS:
            d, s = (np.ascontiguousarray(t) for t in w[name][l])
            keep += [d, s]
            setattr(layers[l], name, _p(d))
            setattr(layers[l], "s" + name[1], _p(s))
        an = np.ascontiguousarray(w["attn_norm"][l], np.float32)
        fn = np.ascontiguousarray(w["ffn_norm"][l], np.float32)
        keep += [an, fn]
        layers[l].attn_norm, layers[l].ffn_norm = _p(an), _p(fn)
    emb = np.ascontiguousarray(w["embedding"], np.float32)
    lm = np.ascontiguousarray(w["lm_head"], np.float32)
    fnorm = np.ascontiguousarray(w["final_norm"], np.float32)
    check(lib().aaedn_abn_model_write(str(path).encode(), ctypes.byref(c), layers, _p(emb), _p(fnorm), _p(lm)))


def from_checkpoint(tensors, hf_config=None):
    """(cfg, weights) of a Llama-style checkpoint's tensors."""
    hc = hf_config or {}
    emb = tensors.get("model.embed_tokens.weight")
    if emb is None:
        raise ValueError("missing model.embed_tokens.weight")
    V, D = emb.shape
    L = 0
    while f"model.layers.{L}.self_attn.q_proj.weight" in tensors:
        L += 1
    if L == 0:
        raise ValueError("no model.layers.<l>.self_attn.q_proj.weight")
    H = int(hc.get("num_attention_heads", D // 128))
    KV = int(hc.get("num_key_value_heads", H))
    hd = D // H
    F = tensors["model.layers.0.mlp.gate_proj.weight"].shape[0]
    cfg = dict(dim=D, n_layers=L, n_heads=H, n_kv_heads=KV, head_dim=hd, ffn_dim=F, vocab=V, max_seq=0,
               rope_theta=float(hc.get("rope_theta", 10000.0)), eps=float(hc.get("rms_norm_eps", 1e-6)))
    names = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj",
             "wo": "self_attn.o_proj", "wg": "mlp.gate_proj", "wu": "mlp.up_proj", "wd": "mlp.down_proj"}
    w = {k: [] for k in LAYER_MATS}
    w["attn_norm"], w["ffn_norm"] = [], []
    for l in range(L):
        pre = f"model.layers.{l}."
        for k, n in names.items():
            w[k].append(quantize_q4(tensors[pre + n + ".weight"]))
        w["attn_norm"].append(tensors[pre + "input_layernorm.weight"].astype(np.float32))
        w["ffn_norm"].append(tensors[pre + "post_attention_layernorm.weight"].astype(np.float32))
    w["embedding"] = emb.astype(np.float32)
    w["lm_head"] = tensors.get("lm_head.weight", emb).astype(np.float32)
    w["final_norm"] = tensors.get("model.norm.weight", np.ones(D, np.float32)).astype(np.float32)
    return cfg, w


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--model", required=True, help="input .safetensors")
    ap.add_argument("--config", default=None, help="Hugging Face config.json (heads, KV heads, theta, eps)")
    ap.add_argument("--output", required=True, help="output .abn")
    a = ap.parse_args(argv)
    hc = None
    if a.config:
        with open(a.config) as f:
            hc = json.load(f)
    cfg, w = from_checkpoint(read_safetensors(a.model), hc)
    write_abn_model(a.output, cfg, w)
    print(f"wrote {a.output}: {cfg['n_layers']} layers, dim {cfg['dim']}, {cfg['n_heads']} heads "
          f"({cfg['n_kv_heads']} KV), ffn {cfg['ffn_dim']}, vocab {cfg['vocab']}, {os.path.getsize(a.output)} bytes")


if __name__ == "__main__":
    main()
