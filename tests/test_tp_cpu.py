"""Tensor parallelism on CPU: two gloo ranks take their shares of a layer by
the library's own plan (aaedn_tp_plan_get), compute them from the
block-quantized weights, and combine them the way the GPU ranks do
(column-parallel qkv and gate/up, row-parallel o and down summed over the
ranks, lm_head rows with an argmax exchange). The combination must equal
the unsharded computation. No GPU is used."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import aaedn_b200 as ab

CFG = dict(dim=256, n_layers=1, n_heads=8, n_kv_heads=4, head_dim=32, ffn_dim=512, vocab=1000, max_seq=64,
           rope_theta=10000.0, eps=1e-6)


def _deq(q, rows, cols):
    d, s = q
    c = np.stack([d & 15, d >> 4], 1).reshape(-1).astype(np.float64)
    return (c * np.repeat(s.view(np.float16).astype(np.float64), 32)).reshape(rows, cols)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, size, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=size)
    try:
        cfg = CFG
        D, hd, H, KV, F, V = (cfg[k] for k in ("dim", "head_dim", "n_heads", "n_kv_heads", "ffn_dim", "vocab"))
        w = ab.synthetic_weights(cfg, 5)
        p = ab.tp_plan(cfg, rank, size)
        rng = np.random.default_rng(0)  # the same inputs on every rank
        x = rng.normal(0, 1, D)
        attn = rng.normal(0, 1, H * hd)
        hid = rng.normal(0, 1, D)
        Wq, Wk, Wv = _deq(w["wq"][0], H * hd, D), _deq(w["wk"][0], KV * hd, D), _deq(w["wv"][0], KV * hd, D)
        Wo, Wg, Wu, Wd = (_deq(w["wo"][0], D, H * hd), _deq(w["wg"][0], F, D), _deq(w["wu"][0], F, D),
                          _deq(w["wd"][0], D, F))
        q0, k0, f0 = p["q_head0"] * hd, p["kv_head0"] * hd, p["ffn_row0"]
        nq, nk, nf = p["n_heads"] * hd, p["n_kv_heads"] * hd, p["ffn_dim"]
        # column-parallel qkv: the ranks' rows side by side are the whole output
        mine = np.concatenate([Wq[q0:q0 + nq] @ x, Wk[k0:k0 + nk] @ x, Wv[k0:k0 + nk] @ x])
        parts = [torch.zeros(mine.size, dtype=torch.float64) for _ in range(size)]
        dist.all_gather(parts, torch.from_numpy(mine))
        parts = [t.numpy() for t in parts]
        got_q = np.concatenate([pp[:nq] for pp in parts])
        got_k = np.concatenate([pp[nq:nq + nk] for pp in parts])
        ok = np.allclose(got_q, Wq @ x, rtol=1e-12) and np.allclose(got_k, Wk @ x, rtol=1e-12)
        # row-parallel o: partial sums over the rank's input columns, summed
        part = torch.from_numpy(Wo[:, q0:q0 + nq] @ attn[q0:q0 + nq])
        dist.all_reduce(part)
        ok = ok and np.allclose(part.numpy(), Wo @ attn, rtol=1e-9, atol=1e-12)
        # gate/up rows, SwiGLU, row-parallel down
        g, u = Wg[f0:f0 + nf] @ hid, Wu[f0:f0 + nf] @ hid
        act = g / (1 + np.exp(-g)) * u
        part = torch.from_numpy(Wd[:, f0:f0 + nf] @ act)
        dist.all_reduce(part)
        G, U = Wg @ hid, Wu @ hid
        ok = ok and np.allclose(part.numpy(), Wd @ (G / (1 + np.exp(-G)) * U), rtol=1e-9, atol=1e-12)
        # lm_head rows and the argmax exchange (ties to the lowest id)
        lm = w["lm_head"].astype(np.float64)
        v0, nv = p["vocab0"], p["vocab"]
        lg = lm[v0:v0 + nv] @ hid
        best = torch.tensor([lg.max(), v0 + int(lg.argmax())], dtype=torch.float64)
        allb = [torch.zeros(2, dtype=torch.float64) for _ in range(size)]
        dist.all_gather(allb, best)
        vals = [(b[0].item(), int(b[1].item())) for b in allb]
        tok = min(vals, key=lambda t: (-t[0], t[1]))[1]
        ok = ok and tok == int((lm @ hid).argmax())
        q.put((rank, bool(ok), p))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("size", [2, 4])
def test_tp_shares_recombine_to_the_whole_layer(size):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, size, port, q)) for r in range(size)]
    for pr in procs:
        pr.start()
    res = [q.get(timeout=300) for _ in range(size)]
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    res.sort()
    assert all(ok for _, ok, _ in res), res
    # the plans tile the model: heads, kv heads, ffn rows, vocabulary
    plans = [p for _, _, p in res]
    for key, n, start in (("n_heads", "n_heads", "q_head0"), ("n_kv_heads", "n_kv_heads", "kv_head0"),
                          ("ffn_dim", "ffn_dim", "ffn_row0"), ("vocab", "vocab", "vocab0")):
        starts = [p[start] for p in plans]
        assert starts == sorted(starts) and starts[0] == 0
        assert all(plans[i][start] + plans[i][key] == (plans[i + 1][start] if i + 1 < size else CFG[n])
                   for i in range(size))


def test_tp_plan_rejects_shapes_that_do_not_divide():
    bad = dict(CFG, n_kv_heads=3, n_heads=3)
    with pytest.raises(ab.AaednError):
        ab.tp_plan(bad, 0, 2)
    with pytest.raises(ab.AaednError):
        ab.tp_plan(CFG, 0, 3)
    p = ab.tp_plan(dict(ab.LLAMA2_7B), 7, 8)
    assert p["ffn_dim"] == 1376 and p["down_k"] == 1408 and p["o_k"] == 512 and p["vocab0"] == 28000


@pytest.mark.parametrize("size", [2, 4, 8])
def test_tp_plan_7b_shares(size):
    """The 7B shape splits at 2, 4 and 8 ranks: heads, kv heads, FFN rows and
    vocabulary rows tile the whole without overlap, and the row-parallel
    input widths (o, down) are padded to whole 128-code tiles (11008 / 4 =
    2752 FFN columns per rank -> 2816), which the tile-major GEMV needs."""
    cfg = dict(ab.LLAMA2_7B)
    plans = [ab.tp_plan(cfg, r, size) for r in range(size)]
    assert sum(p["n_heads"] for p in plans) == cfg["n_heads"]
    assert sum(p["n_kv_heads"] for p in plans) == cfg["n_kv_heads"]
    assert sum(p["ffn_dim"] for p in plans) == cfg["ffn_dim"]
    assert sum(p["vocab"] for p in plans) == cfg["vocab"]
    for r, p in enumerate(plans):
        assert p["q_head0"] == r * p["n_heads"] and p["kv_head0"] == r * p["n_kv_heads"]
        assert p["ffn_row0"] == r * p["ffn_dim"]
        assert p["o_k"] % 128 == 0 and p["o_k"] >= p["n_heads"] * cfg["head_dim"]
        assert p["down_k"] % 128 == 0 and p["down_k"] >= p["ffn_dim"] and p["down_k"] - p["ffn_dim"] < 128
    assert [p["vocab0"] for p in plans] == list(np.cumsum([0] + [p["vocab"] for p in plans[:-1]]))
