#!/usr/bin/env python3
"""Decode benchmark of the token loop on B200.

Workload: the Llama-2-7B-shaped block-quantized random model (dim 4096, 32
layers, 32 heads x 128, SwiGLU 11008, vocab 32000, ctx 4096), a 128-token
seeded uniform-random prompt, then greedy decode at batch 1. A step is one
decode token (one pass of the whole token loop). Weights are N(0, 0.02)
from the seeded generator, quantized with the reference's block quantizer;
there is no dataset (data: synthetic).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Ours: W untimed device-resident decode steps, then exactly K timed steps
(CUDA events on the model's stream, barrier + synchronize on both sides, max
over ranks). Under torchrun the N ranks decode ONE sequence tensor-parallel
(heads, FFN rows and lm_head rows sharded; partial sums added through peer
memory over NVLink; strong scaling), or with --mode replicas N independent
sequences (weak scaling).
The line also carries the end-to-end rate through the reference-facing
call (transformer_forward semantics: host token in, host logits out, host
argmax), the roofline of the dequant-GEMV kernels from CUDA events, the SM
clocks sampled during the timed region and the CPU baseline (the oracle
restatement on the host cores, rank 0 only).

Reference arm (--impl reference): the reference's CPU token loop cannot run
end to end (src/transformer.cpp:156 overflows a static buffer), so the arm
times the CPU restatement of that loop (oracle/, built with the reference's
own flags) on all host threads, on a bounded sample of the same workload:
the same weights (the oracle's restatement of the seeded generator and of
the block quantizer), decode steps from the same first position. It loads
nothing of this repository's CUDA library.

Parity: when the workload is the full 7B model with the 128-token prompt,
the first 32 greedy tokens of the run (every N, tensor parallel included)
are compared with the oracle's (tests/golden/llama2_7b_seed1234.npz) and the
line carries "parity": true/false.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "project-aaedn_b200"))

METRIC = "decode tok/s (7B-shape, bs1, 1 GPU) + dequant-GEMV GB/s vs HBM peak"
SEED = 1234
PROMPT = 128
FALLBACK_HBM_GBS = 6650.0
# the Llama-2-7B-shaped model (both arms; the reference arm must not import
# the CUDA library's package for it)
LLAMA2_7B = dict(dim=4096, n_layers=32, n_heads=32, n_kv_heads=32, head_dim=128, ffn_dim=11008, vocab=32000,
                 max_seq=4096, rope_theta=10000.0, eps=1e-6)
PARITY_FIXTURE = os.path.join(ROOT, "tests", "golden", "llama2_7b_seed1234.npz")
PARITY_TOKENS = 32
PARITY_LOGITS_TOL = 1e-3  # relative max-abs on the logits after the prompt (the task's bar is 1e-2)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=512)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=None,
                    help="end-to-end steps (default: --steps, over the timed region's positions)")
    ap.add_argument("--profile-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=20.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-microbench", action="store_true", help="skip the dequant-GEMV/GEMM microbenchmark")
    ap.add_argument("--workload", default="decode", choices=["decode", "batched"],
                    help="decode: the headline 7B bs1 decode; batched: the 8B-GQA batched decode (its own line)")
    ap.add_argument("--batch", type=int, default=32, help="batched workload: streams")
    ap.add_argument("--batch-prompt", type=int, default=2048, help="batched workload: prompt tokens per stream")
    ap.add_argument("--mode", default="tp", choices=["tp", "replicas"],
                    help="N > 1 GPUs: one sequence tensor-parallel over the N GPUs (strong scaling), or N "
                         "independent replicas (weak scaling)")
    # smaller cases of the same model for profiler captures (not bench lines)
    ap.add_argument("--layers", type=int, default=None, help="profiling case: fewer layers than the 7B model")
    ap.add_argument("--prompt", type=int, default=PROMPT, help="profiling case: prompt length")
    ap.add_argument("--ctx", type=int, default=None, help="profiling case: context length")
    return ap.parse_args()


def model_cfg(args=None):
    cfg = dict(LLAMA2_7B)
    if args is not None and args.layers:
        cfg["n_layers"] = args.layers
    if args is not None and args.ctx:
        cfg["max_seq"] = args.ctx
    return cfg


def gemv_shapes(cfg):
    D, H, hd, KV, F = cfg["dim"], cfg["n_heads"], cfg["head_dim"], cfg["n_kv_heads"], cfg["ffn_dim"]
    # (rows, cols) of the four dequant-GEMVs of one layer, in launch order
    return {"qkv": ((H + 2 * KV) * hd, D), "o": (D, H * hd), "gate_up": (2 * F, D), "down": (D, F)}


def gemv_bytes(n, k, m=1):
    """Algorithmic bytes of one M-row dequant-GEMV: codes + fp16 scales
    (0.5625 B/weight) + fp32 activations in and out."""
    return n * k * 0.5625 + 4 * (m * k + m * n)


def step_bytes(cfg, pos):
    """Algorithmic bytes of one decode step at position pos: every weight
    once, the fp32 lm_head, and the K/V rows of positions 0..pos."""
    w = sum(gemv_bytes(n, k) for n, k in gemv_shapes(cfg).values()) * cfg["n_layers"]
    lm = cfg["vocab"] * cfg["dim"] * 4
    kv = cfg["n_layers"] * 2 * (pos + 1) * cfg["n_kv_heads"] * cfg["head_dim"] * 4
    return w + lm + kv


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """dram bytes per GEMV launch from the committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", "gemv_tiled_i8_decode_7b.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch_avg:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons of one GPU while running."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(gpu_id)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in out.strip().splitlines():
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_identity(dev_index):
    import torch
    try:
        p = torch.cuda.get_device_properties(dev_index)
        bus = getattr(p, "pci_bus_id", None)
        dom = getattr(p, "pci_domain_id", 0)
        dv = getattr(p, "pci_device_id", 0)
        if bus is not None:
            return f"{dom:08x}:{bus:02x}:{dv:02x}.0"
    except Exception:
        pass
    return str(dev_index)


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def oracle_weights(cfg):
    """The seeded synthetic model built by the oracle alone (bit-identical to
    the library's aaedn_model_synthesize, tests/test_oracle_golden.py)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle
    o = pyoracle.Oracle()
    o.set_threads(host_cores())
    return pyoracle.synthetic_weights(cfg, SEED, o)


def cpu_decode_sample(cfg, w, seconds, pos0, steps_cap=None, warmup=1):
    """Times greedy decode steps of the CPU restatement (oracle/, reference
    flags, every host core) from position pos0 (the cache below it filled by
    the oracle's seek), `warmup` untimed steps first; returns (tok/s, steps,
    threads, description)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle
    orc = pyoracle.Oracle(fast=True)
    # torch.distributed.run exports OMP_NUM_THREADS=1: the CPU arm sets its
    # thread count itself
    orc.set_threads(host_cores())
    n_ctx = pos0 + warmup + (steps_cap or 256) + 2
    c = dict(cfg, max_seq=min(cfg["max_seq"], max(256, n_ctx)))
    om = pyoracle.OracleModel(orc, c, w)
    om.seek(pos0)
    tok = int(orc.synth_tokens(SEED, 0, cfg["vocab"], 1)[0])
    for _ in range(max(1, warmup)):
        tok = int(np.argmax(om.step(tok)))
    t0 = time.perf_counter()
    logits = om.step(tok)
    first = time.perf_counter() - t0
    n = max(1, min(int(seconds / max(first, 1e-3)), steps_cap or 10 ** 9, c["max_seq"] - om.pos - 1))
    t0 = time.perf_counter()
    for _ in range(n):
        tok = int(np.argmax(logits))
        logits = om.step(tok)
    dt = time.perf_counter() - t0
    p1 = om.pos
    desc = (f"{n} greedy decode steps of the full {cfg['n_layers']}-layer 7B-shape model at positions "
            f"{p1 - n}..{p1 - 1} (the GPU arm's first timed position {pos0}; K/V below it from the oracle's "
            f"seek), oracle built -O3 -mavx2 -mfma -ffast-math, OpenMP over GEMV rows and heads on "
            f"{orc.threads()} threads")
    cpu_decode_sample.last_positions = [p1 - n, p1]
    return n / dt, n, orc.threads(), desc


def workload_config(cfg, args, positions=None, parallelism="single GPU"):
    full = (cfg["n_layers"], args.prompt) == (32, PROMPT)
    return {"workload": ("llama2-7b-shape q4 greedy decode bs1: 128-token prompt, then decode" if full else
                         f"profiling case: {cfg['n_layers']} layers, {args.prompt}-token prompt"),
            "dim": cfg["dim"], "n_layers": cfg["n_layers"], "n_heads": cfg["n_heads"],
            "head_dim": cfg["head_dim"], "ffn_dim": cfg["ffn_dim"], "vocab": cfg["vocab"],
            "ctx": cfg["max_seq"], "prompt": args.prompt,
            "positions": positions if positions is not None else [args.prompt + max(3, args.warmup),
                                                                  args.prompt + max(3, args.warmup) + args.steps],
            "weights": "4-bit codes, fp16 scale per 32, fp32 embedding/lm_head",
            "l2": "inputs larger than L2: 4.1 GB of weights streamed per step",
            "parallelism": parallelism}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cfg = model_cfg(args)
    if not os.path.exists(os.path.join(ROOT, "oracle", "build", "liboracle_fast.so")):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "oracle"], check=True, capture_output=True)
    w = oracle_weights(cfg)
    # the GPU arm's timed region starts after the prompt and W warm-up steps;
    # each step here is one decode token from there, the count bounded so the
    # run stays within a few minutes of CPU time
    W = max(3, args.warmup)
    pos0 = args.prompt + W
    cap = max(1, args.steps)
    value, n, threads, desc = cpu_decode_sample(cfg, w, seconds=max(5.0, args.cpu_seconds), pos0=pos0,
                                                steps_cap=cap)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": n, "warmup": 1, "ms_per_step": 1000.0 / value, "higher_is_better": True,
        "scaling": "strong" if args.gpus > 1 else "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": dict(workload_config(cfg, args, positions=cpu_decode_sample.last_positions,
                                       parallelism=f"CPU, {threads} threads"),
                       sample=f"{n} decode steps against the GPU arm's {args.steps}, from its first timed "
                              f"position {pos0} (+ the warm-up step)"),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def measured_bf16_tflops():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def prefill_report(cfg, n, ms, shards, chunk_rows):
    """The prompt's prefill: tokens/s, the linear layers' algorithmic
    TFLOP/s (2 M N K per matrix) and the tensor-pipe TFLOP/s they cost (five
    bf16 MMAs per fp32 multiply-add: the three activation parts times the
    two exact weight parts above 2^-24) against the bf16 peak. The time
    includes attention, norms and the lm_head of the last token."""
    lin = sum(r * k for r, k in gemv_shapes(cfg).values()) * cfg["n_layers"] / shards
    alg = 2.0 * n * lin / (ms / 1000.0) / 1e12
    peak, kind = measured_bf16_tflops()
    return {"tokens": n, "ms": ms, "tok_s": n / (ms / 1000.0), "linear_tflops": alg,
            "tensor_pipe_tflops": 5 * alg, "tensor_peak_tflops": peak, "tensor_frac": 5 * alg / peak,
            "peak_kind": kind,
            "path": ("tcgen05 GEMM (TMEM accumulators, TMA-fed activation parts)" if chunk_rows else
                     "one decode step per prompt token")}


def microbench(reps=20):
    """The dequant-GEMV / GEMM microbenchmark on the block-quant format
    (weights N(0, 0.02) quantized, activations N(0, 1) fp32): shapes
    4096x4096, 11008x4096, 4096x11008 at M = 1, 8 and 64, through
    fused_matmul on the reference's row-major layout (M <= 8: the row-major
    GEMV; M = 64: tcgen05 GEMM) and through fused_matmul_tiled on the
    model's tile-major repacking of the same blocks (M = 1: the decode GEMV
    engine; M = 8, 64: tcgen05 GEMM). GB/s of codes + scales + activations
    against the HBM peak, TFLOP/s as 2 M N K. Enough weight copies rotate
    that every call reads HBM (more than the 126 MB of L2)."""
    import torch
    import aaedn_b200 as ab
    peak, _ = measured_peaks()
    out = []
    for N, K in ((4096, 4096), (11008, 4096), (4096, 11008)):
        wbytes = N * K // 2 + N * K // 16
        copies = max(2, int(400e6 // wbytes) + 1)
        d, sc = ab.quantize_q4(ab.synth_normal(77, N + K, N * K))
        wd = torch.from_numpy(d).cuda()
        ws = torch.from_numpy(sc.view(np.int16)).cuda()
        W = [(wd.clone(), ws.clone()) for _ in range(copies)]
        for M in (1, 8, 64):
            x = torch.from_numpy(ab.synth_normal(78, M, M * K, std=1.0)).cuda()
            y = torch.empty(M * N, dtype=torch.float32, device="cuda")
            for i in range(3):
                ab.fused_matmul(x, W[i % copies][0], W[i % copies][1], y, M, N, K)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for i in range(reps):
                ab.fused_matmul(x, W[i % copies][0], W[i % copies][1], y, M, N, K)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            byts = gemv_bytes(N, K, M)
            row = {"N": N, "K": K, "M": M, "layout": "row-major", "us": ms * 1e3, "gbs": byts / (ms / 1e3) / 1e9,
                   "hbm_frac": byts / (ms / 1e3) / 1e9 / peak, "tflops": 2.0 * M * N * K / (ms / 1e3) / 1e12,
                   "engine": "tcgen05 GEMM" if M > 8 else "GEMV (mma.sync bf16, three activation parts)"}
            out.append(row)
        del W
        # the same weights in the model's tile-major layout: M = 1 on the
        # decode GEMV engine, M = 8 and 64 on the tcgen05 GEMM
        tiled = torch.from_numpy(ab.repack_tiled(d, sc, N, K)).cuda()
        T = [tiled.clone() for _ in range(copies)]
        for M in (1, 8, 64):
            x = torch.from_numpy(ab.synth_normal(78, M, M * K, std=1.0)).cuda()
            y = torch.empty(M * N, dtype=torch.float32, device="cuda")
            for i in range(3):
                ab.fused_matmul_tiled(x, T[i % copies], y, M, N, K)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for i in range(reps):
                ab.fused_matmul_tiled(x, T[i % copies], y, M, N, K)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            byts = gemv_bytes(N, K, M)
            out.append({"N": N, "K": K, "M": M, "layout": "tile-major", "us": ms * 1e3,
                        "gbs": byts / (ms / 1e3) / 1e9, "hbm_frac": byts / (ms / 1e3) / 1e9 / peak,
                        "tflops": 2.0 * M * N * K / (ms / 1e3) / 1e12,
                        "engine": "decode GEMV (integer MMA over activation digits)" if M == 1 else "tcgen05 GEMM"})
        del T, tiled
    return out


def parity_check(model, cfg, args, tp, prompt_logits):
    """The run's first greedy tokens and its logits after the prompt against
    the oracle fixture of the full 7B model (None when the workload is not
    that model). A tensor-parallel rank compares its slice of the logits."""
    if (cfg["n_layers"], args.prompt) != (32, PROMPT) or not os.path.exists(PARITY_FIXTURE):
        return None
    fx = np.load(PARITY_FIXTURE)
    wl = fx["logits_prompt"]
    lo, n = (model.tp_share() if tp else (0, cfg["vocab"]))
    lerr = float(np.abs(prompt_logits[lo:lo + n] - wl[lo:lo + n]).max() / np.abs(wl).max())
    want = fx["tokens"][:PARITY_TOKENS]
    have = model.pos - args.prompt + 1  # greedy tokens produced since the prompt
    if have < PARITY_TOKENS:
        model.decode_steps(PARITY_TOKENS - have)
    got = model.tokens(PARITY_TOKENS)
    bad = np.nonzero(got != want)[0]
    return {"match": bool(bad.size == 0) and lerr <= PARITY_LOGITS_TOL, "tokens": PARITY_TOKENS,
            "first_mismatch": int(bad[0]) if bad.size else None, "logits_rel_err": lerr,
            "logits_tol": PARITY_LOGITS_TOL,
            "against": "tests/golden/llama2_7b_seed1234.npz (strict oracle, seed 1234)"}


def run_ours(args):
    import torch
    import torch.distributed as dist
    import aaedn_b200 as ab

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    cfg = model_cfg(args)
    K, W = args.steps, max(3, args.warmup)
    E, P = (args.e2e_steps if args.e2e_steps is not None else K), args.profile_steps
    if args.prompt + W + max(K, E) + P + 2 > cfg["max_seq"]:
        raise SystemExit(f"steps+warmup too large for ctx {cfg['max_seq']}")

    tp = world > 1 and args.mode == "tp"
    model = ab.Model(cfg, tp=(rank, world) if tp else None)
    model.synthesize(SEED)  # the seeded synthetic model, generated and quantized on the host, uploaded
    if tp:
        model.connect_tp()
    stream = torch.cuda.ExternalStream(model.stream)
    prompt = ab.synth_tokens(SEED, 0, cfg["vocab"], args.prompt)

    # prefill: the prompt's tokens together through the tensor-core GEMMs
    # (timed on the model's stream after one untimed prefill of the same
    # prompt), then W warm-up decode steps
    model.forward(prompt, want_logits=False)
    model.reset()
    pf0, pf1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    pf0.record(stream)
    model.forward(prompt, want_logits=False)
    pf1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = pf0.elapsed_time(pf1)
    prompt_logits = model.logits()  # this rank's vocabulary slice (the rest zero)
    model.decode_steps(W)
    torch.cuda.synchronize()
    pos0 = model.pos

    # ---- timed region: exactly K device-resident greedy steps
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(gpu_identity(local))
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    launches0 = ab.kernel_launches()
    ev0.record(stream)
    model.decode_steps(K)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    launches = ab.kernel_launches() - launches0
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    # the run's first greedy tokens against the oracle (outside the timed
    # region; every rank takes the same steps)
    parity = parity_check(model, cfg, args, tp, prompt_logits)
    if parity is not None and world > 1:
        # every rank checked its slice of the logits: the worst over ranks
        t = torch.tensor([parity["logits_rel_err"]], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        parity["logits_rel_err"] = float(t.item())
        parity["match"] = parity["match"] and parity["logits_rel_err"] <= PARITY_LOGITS_TOL
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    streams = 1 if tp else world  # tensor parallel: the N GPUs decode one sequence
    value = streams * K / (ms_max / 1000.0)
    pos1 = model.pos

    # ---- end to end through the reference-facing call (host token in, host
    # logits out, host argmax), E steps from the timed region's first
    # position (the sequence restarted: the same prompt and warm-up steps,
    # untimed); the token and the logits live in pinned host buffers
    model.reset()
    model.forward(prompt, want_logits=False)
    model.decode_steps(W)
    torch.cuda.synchronize()
    assert model.pos == pos0
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, pin_memory=True).numpy()
    logits[:] = model.logits()
    tok = torch.empty(1, dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(E):
        # tensor parallel: each rank holds a vocabulary slice of the logits;
        # the ranks' argmax exchange already chose the token on the device
        tok[0] = model.next_token() if tp else int(np.argmax(logits))
        model.forward(tok, out=logits)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    te = torch.tensor([e2e_ms], device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = streams * E / (float(te.item()) / 1000.0)

    # ---- per-kernel-class device times: sub-graphs of the decode step (only
    # the dequant-GEMVs, only attention, ...) replayed P times back to back,
    # so the figures carry the same launch overlap as the decode graph and no
    # event overhead between kernels
    L = cfg["n_layers"]
    if tp:
        # a part of a tensor-parallel step alone would wait for partials its
        # peers never send: the split is taken from whole steps (per-kernel
        # events, no launch overlap)
        pk = np.stack([model.profile_step() for _ in range(max(1, P))]).mean(0)
        # entries: per layer qkv, attention, o, gate/up, down (the last down
        # with the final reduction); then lm_head with the argmax exchange
        n5 = 5 * L
        parts = {"step": float(pk.sum()), "lm_head": float(pk[n5])}
        lay = pk[:n5].reshape(L, 5)
        for i, k in enumerate(("qkv", "attention", "o", "gate_up", "down")):
            parts[k] = float(lay[:, i].sum())
        parts["gemv"] = parts["qkv"] + parts["o"] + parts["gate_up"] + parts["down"]
    else:
        parts = model.profile_parts(reps=P)
    shapes = gemv_shapes(cfg)
    gemv_total_ms = parts["gemv"]
    gemv_total_bytes = sum(gemv_bytes(*shapes[k]) for k in ("qkv", "o", "gate_up", "down"))
    # tensor parallel: each GPU streams its 1/N share of every matrix
    share = 1.0 / world if tp else 1.0
    achieved = gemv_total_bytes * share * L / (gemv_total_ms / 1000.0) / 1e9
    peak, peak_kind = measured_peaks()
    kernel_split = {"step_ms": parts["step"], "gemv_ms": parts["gemv"], "attention_ms": parts["attention"],
                    "lm_head_ms": parts["lm_head"],
                    **{f"{k}_ms": parts[k] for k in ("qkv", "o", "gate_up", "down")},
                    **{f"{k}_gbs": gemv_bytes(*shapes[k]) * share * L / (parts[k] / 1000.0) / 1e9
                       for k in ("qkv", "o", "gate_up", "down")},
                    "lm_head_gbs": cfg["vocab"] * cfg["dim"] * 4 * share / (parts["lm_head"] / 1000.0) / 1e9}
    traffic = profiled_traffic()

    mean_pos = (pos0 + pos1 - 1) / 2.0
    sb = step_bytes(cfg, mean_pos) * share  # per GPU
    step_gbs = sb / (ms_max / K / 1000.0) / 1e9

    micro = None
    if rank == 0 and world == 1 and not args.no_microbench:
        try:
            micro = microbench()
        except Exception as ex:  # the decode number stands without it
            micro = [{"failed": str(ex)}]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            v, n, threads, desc = cpu_decode_sample(cfg, oracle_weights(cfg), args.cpu_seconds, pos0=pos0)
            cpu = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port", "sample": desc}
        except Exception as ex:  # the GPU number stands without it
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "port", "sample": f"failed: {ex}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "strong" if tp else "weak",
            "vs_baseline": None,
            "dtype": "fp32", "data": "synthetic",
            "config": workload_config(cfg, args, positions=[pos0, pos1],
                                      parallelism=(f"tp{world} (heads, ffn rows, lm_head rows; partials added "
                                                   "over NVLink peer memory)" if tp else
                                                   f"replicas x{world}" if world > 1 else "single GPU")),
            "parity": None if parity is None else parity["match"],
            "parity_detail": parity,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": "gemv_tiled_i8_kernel (the 4 dequant-GEMVs of every layer, M=1)",
                         "launches_per_step": 4 * L, "bytes_per_launch_avg": gemv_total_bytes * share / 4,
                         "bytes_per_step": gemv_total_bytes * share * L,
                         "timing": ("per-kernel CUDA events inside whole steps" if tp else
                                    "sub-graph of the step's GEMVs replayed back to back, CUDA events")},
            "decode_step": {"algorithmic_bytes": sb, "achieved_gbs": step_gbs, "frac": step_gbs / peak,
                            **kernel_split},
            "prefill": prefill_report(cfg, args.prompt, prefill_ms, world if tp else 1, model.prefill_rows),
            "microbench": micro,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 12,
                    "d2h_bytes_per_step": (4 * ab.tp_plan(cfg, rank, world)["vocab"] + 4) if tp else 4 * cfg["vocab"],
                    "call": ("aaedn_model_forward (transformer_forward, this rank's logits slice) + the "
                             "device's next token" if tp else
                             "aaedn_model_forward (transformer_forward) + host argmax"),
                    "steps": E, "positions": [pos0, pos0 + E]},
            "gpu_launches": int(launches),
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    barrier()  # tensor parallel: no rank frees memory a peer may still read
    model.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


LLAMA3_8B = dict(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128, ffn_dim=14336, vocab=128256,
                 max_seq=4096, rope_theta=500000.0, eps=1e-6)


def run_batched(args):
    """The Llama-3-8B-shaped GQA model with a batch of streams (default 32),
    each prefilled with its own seeded random prompt (default 2048 tokens),
    then decoded together at batch width (default 256 steps): one GPU, the
    batched model (shared paged KV pool, tensor-core GEMMs over the batch).
    Prints one JSON line of its own (not the headline metric)."""
    import torch
    import aaedn_b200 as ab
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    B, T, K, W = args.batch, args.batch_prompt, args.steps, max(3, args.warmup)
    cfg = dict(LLAMA3_8B, max_seq=T + W + K + 8)
    if args.layers:
        cfg["n_layers"] = args.layers
    model = ab.BatchedModel(cfg, max_seqs=B, kv_tokens=B * (cfg["max_seq"] + 64))
    t0 = time.time()
    model.synthesize(SEED)
    synth_s = time.time() - t0
    stream = torch.cuda.ExternalStream(model.stream)
    seqs, nxt = [], []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(B):
        s = model.open()
        _, n = model.prefill(s, ab.synth_tokens(SEED, 100 + i, cfg["vocab"], T), want_logits=False)
        seqs.append(s)
        nxt.append(n)
    e1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = e0.elapsed_time(e1)
    for _ in range(W):
        _, out = model.step(seqs, nxt, want_logits=False)
        nxt = [int(v) for v in out]
    torch.cuda.synchronize()
    clocks = ClockSampler(gpu_identity(int(os.environ.get("LOCAL_RANK", "0"))))
    time.sleep(0.3)
    e0.record(stream)
    for _ in range(K):
        _, out = model.step(seqs, nxt, want_logits=False)
        nxt = [int(v) for v in out]
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    peak, kind = measured_peaks()
    L = cfg["n_layers"]
    wbytes = sum(gemv_bytes(n, k, B) for n, k in gemv_shapes(cfg).values()) * L + cfg["vocab"] * cfg["dim"] * 4
    mean_pos = T + W + (K - 1) / 2.0
    kv = L * 2 * B * (mean_pos + 1) * cfg["n_kv_heads"] * cfg["head_dim"] * 4
    step_s = ms / K / 1000.0
    line = {
        "metric": "batched decode tok/s (Llama-3-8B shape, GQA, 1 GPU)", "value": B * K / (ms / 1000.0),
        "unit": "tok/s", "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
        "dtype": "fp32", "data": "synthetic",
        "config": {"workload": f"llama3-8b-shape q4, {B} streams x {T}-token prompt, then {K} batched decode steps",
                   "dim": cfg["dim"], "n_layers": L, "n_heads": cfg["n_heads"], "n_kv_heads": cfg["n_kv_heads"],
                   "ffn_dim": cfg["ffn_dim"], "vocab": cfg["vocab"], "batch": B, "prompt": T,
                   "kv": "fp32 pages of 64 tokens in a shared pool"},
        "roofline": {"bound": "hbm", "algorithmic_bytes_per_step": wbytes + kv,
                     "achieved": (wbytes + kv) / step_s / 1e9, "peak": peak, "unit": "GB/s",
                     "frac": (wbytes + kv) / step_s / 1e9 / peak, "peak_kind": kind},
        "prefill": {"tokens": B * T, "ms": prefill_ms, "tok_s": B * T / (prefill_ms / 1000.0),
                    "linear_tflops": 2.0 * B * T * sum(n * k for n, k in gemv_shapes(cfg).values()) * L /
                    (prefill_ms / 1000.0) / 1e12},
        "synthesize_s": synth_s, "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    model.close()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "batched":
        return run_batched(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
