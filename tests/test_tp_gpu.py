"""Tensor-parallel decode on 2, 4 and 8 GPUs against the oracle: one process
per GPU, each with its share of the model (aaedn_model_create_tp), partial
sums added through each other's memory. The greedy tokens must equal the
oracle's and the assembled logits must agree within 1e-4 (the same bars as
the single-GPU model tests). Needs 2 (4, 8) GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import aaedn_b200 as ab

pytestmark = pytest.mark.gpu

GQA = dict(dim=256, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=32, ffn_dim=512, vocab=1000, max_seq=200,
           rope_theta=500000.0, eps=1e-6)
W7B = dict(ab.LLAMA2_7B, n_layers=2, max_seq=256)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, size, port, cfg, seed, n_prompt, n_new, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=size, timeout=timedelta(seconds=120))
    try:
        w = ab.synthetic_weights(cfg, seed)
        m = ab.Model(cfg, tp=(rank, size))
        m.set_weights(w)
        m.connect_tp()
        prompt = ab.synth_tokens(seed, 0, cfg["vocab"], n_prompt)
        toks = m.generate(prompt, n_new)
        lg = m.logits()
        p = ab.tp_plan(cfg, rank, size)
        share = lg[p["vocab0"]:p["vocab0"] + p["vocab"]].copy()
        dist.barrier()  # no rank tears down while another still reads its memory
        m.close()
        q.put((rank, toks, p["vocab0"], share))
    finally:
        dist.destroy_process_group()


def _run(cfg, seed, n_prompt, n_new, size=2):
    import torch
    if torch.cuda.device_count() < size:
        pytest.skip(f"needs {size} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, size, port, cfg, seed, n_prompt, n_new, q)) for r in range(size)]
    for pr in procs:
        pr.start()
    res = sorted(q.get(timeout=600) for _ in range(size))
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    toks = [r[1] for r in res]
    for t in toks[1:]:
        np.testing.assert_array_equal(t, toks[0])  # lockstep: one token stream
    logits = np.zeros(cfg["vocab"], np.float32)
    for _, _, v0, share in res:
        logits[v0:v0 + share.size] = share
    return toks[0], logits


@pytest.mark.parametrize("cfg,seed,n_prompt,n_new,size", [
    (GQA, 77, 9, 120, 2),
    (W7B, 2024, 4, 64, 2),
    (W7B, 31, 5, 40, 4),
    (W7B, 31, 5, 40, 8),
])
def test_tp_greedy_identical_to_oracle(oracle, cfg, seed, n_prompt, n_new, size):
    import pyoracle
    got, logits = _run(cfg, seed, n_prompt, n_new, size=size)
    w = ab.synthetic_weights(cfg, seed)
    om = pyoracle.OracleModel(oracle, cfg, w)
    want, wl = om.generate(ab.synth_tokens(seed, 0, cfg["vocab"], n_prompt), n_new)
    np.testing.assert_array_equal(got, want)
    assert float(np.abs(logits - wl).max() / np.abs(wl).max()) < 1e-4


def _rank_timeout(rank, size, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=size, timeout=timedelta(seconds=120))
    try:
        cfg = GQA
        m = ab.Model(cfg, tp=(rank, size))
        m.synthesize(7)
        m.connect_tp()
        m.generate(ab.synth_tokens(7, 0, cfg["vocab"], 4), 3)  # both ranks step together
        dist.barrier()
        rc = ab.OK
        if rank == 0:
            # rank 1 launches nothing: rank 0's waits for its partials run out
            # (bounded) and the step reports it; the GPU stays usable
            m.decode_steps(1)
            try:
                m.status()
            except ab.AaednError as e:
                rc = e.rc
        dist.barrier()  # rank 1 stays mapped until rank 0's step is over
        m.close()
        q.put((rank, rc))
    finally:
        dist.destroy_process_group()


def test_tp_peer_that_does_not_step_times_out():
    """A rank whose peer never launches its step gets AAEDN_ETIMEOUT from the
    bounded flag waits (about 2 s), and both ranks shut down cleanly."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_timeout, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    assert res[0] == ab.ETIMEOUT and res[1] == ab.OK
