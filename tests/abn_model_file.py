"""Writes whole-model .abn files (the layout aaedn_abn_model_read_header
documents: the per-layer order of the reference's docs/mpd.md:497-499,
version 3, n_kv_heads / rope_theta / eps in the reserved header bytes) from
the host weights that aaedn_b200.synthetic_weights returns. Test
infrastructure: the reference's converter does not write this layout yet."""
import struct

import numpy as np

import aaedn_b200 as ab


def payload_parts(cfg, w, bias=None):
    D = cfg["dim"]
    parts = []
    for l in range(cfg["n_layers"]):
        q, k, v = (w[n][l] for n in ("wq", "wk", "wv"))
        qkv_rows = (cfg["n_heads"] + 2 * cfg["n_kv_heads"]) * cfg["head_dim"]
        parts.append(np.asarray(w["attn_norm"][l], np.float32))
        parts.append(np.concatenate([q[0], k[0], v[0]]))   # codes of the q, k, v rows
        parts.append(np.concatenate([q[1], k[1], v[1]]))   # their scales
        parts.append(np.zeros(qkv_rows, np.float32) if bias is None else np.asarray(bias, np.float32))
        for n in ("wo", "wg", "wu", "wd"):
            parts.append(w[n][l][0])
            parts.append(w[n][l][1])
        parts.append(np.asarray(w["ffn_norm"][l], np.float32))
    parts.append(np.asarray(w["final_norm"], np.float32).reshape(D))
    parts.append(np.asarray(w["embedding"], np.float32))
    parts.append(np.asarray(w["lm_head"], np.float32))
    return b"".join(np.ascontiguousarray(p).tobytes() for p in parts)


def header(cfg, payload, version=3, quant_type=0):
    reserved = struct.pack("<Iff3x", cfg["n_kv_heads"], cfg["rope_theta"], cfg["eps"])
    checksum = ab.fnv1a32(np.frombuffer(payload, np.uint8)) if payload else 0
    return struct.pack("<8sIQI6IB", b"AAEDNMDL", version, len(payload), checksum, cfg["n_layers"],
                       cfg["n_heads"], cfg["head_dim"], cfg["vocab"], cfg["dim"], cfg["ffn_dim"],
                       quant_type) + reserved


def write(path, cfg, w, bias=None, version=3):
    payload = payload_parts(cfg, w, bias)
    with open(path, "wb") as f:
        f.write(header(cfg, payload, version))
        f.write(payload)
    return len(payload)
