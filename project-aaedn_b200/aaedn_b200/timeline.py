"""Timeline of one decode step of the per-kernel graph, from the per-CTA
globaltimer stamps of aaedn_model_trace_kernels.

    python -m aaedn_b200.timeline [--layers 32] [--prompt 128] [--decode 200] [--seed 1234]

Builds the Llama-2-7B-shaped model on cuda:0 with weights synthesized on the
device, decodes `--decode` steps after the prompt, traces one step and
prints, per kernel of a layer (averaged over layers 1..L-1): its span (last
exit of the previous kernel to its own last exit), when its CTAs entered,
when the wait for the previous kernel returned, when the operand was built
(GEMVs), and the spread of exits. All times in microseconds.
"""
import argparse

import numpy as np

from . import LLAMA2_7B, Model, synth_tokens

NAMES = ("qkv", "attention", "o", "gate_up", "down")


def layer_table(stamps, grid, n_layers):
    """Per kernel of a layer, the mean over layers 1..L-1 of: span, entry
    (first, median) and exit (median, last) relative to the previous
    kernel's last exit, and (GEMVs) wait-done and operand-ready medians."""
    rows = {n: [] for n in NAMES}
    st = stamps.astype(np.int64)
    prev_exit = None
    for k in range(5 * n_layers):
        g = int(grid[k])
        if g == 0:
            prev_exit = None
            continue
        s = st[k, :g]
        ent, ev1, ev2, ext = s[:, 0], s[:, 1], s[:, 2], s[:, 3]
        if prev_exit is not None and k >= 5:
            r = {"span": ext.max() - prev_exit, "entry_first": ent.min() - prev_exit,
                 "entry_med": np.median(ent) - prev_exit, "exit_med": np.median(ext) - prev_exit,
                 "exit_last": ext.max() - prev_exit}
            if k % 5 != 1:  # GEMV: 2 = wait returned, 1 = operand built
                r["wait_done"] = np.median(ev2) - prev_exit
                r["ready"] = np.median(ev1) - prev_exit
            else:  # attention: 1 = wait returned, 2 = token loop done
                r["wait_done"] = np.median(ev1) - prev_exit
                r["ready"] = np.median(ev2) - prev_exit
            rows[NAMES[k % 5]].append(r)
        prev_exit = ext.max()
    return {n: {key: float(np.mean([r[key] for r in v])) / 1e3 for key in v[0]} for n, v in rows.items() if v}


CHUNK_CTAS, CHUNKS = 8, 24  # per-chunk stamps of a tiled GEMV's first CTAs


def chunk_view(stamps, grid, layer, events_per_cta, chunk_base, n_kv):
    """Per GEMV of `layer`: for its first CTAs, entry / wait / ready / exit and
    each chunk's consumer start-end; for the attention, the CTAs of kv head
    0's splits (one cluster). us from the previous kernel's last exit."""
    st = stamps.astype(np.int64)
    flat = st.reshape(st.shape[0], -1)
    lines = []
    ka = 5 * layer + 1
    prev = st[ka - 1, :int(grid[ka - 1]), 3].max()
    lines.append(f"attention (layer {layer}), kv head 0: split entry wait ready exit")
    for sp in range(int(grid[ka]) // n_kv):
        ev = (st[ka, sp * n_kv] - prev) / 1e3
        lines.append(f"  split {sp}: {ev[0]:.2f} {ev[1]:.2f} {ev[2]:.2f} {ev[3]:.2f}")
    for j, name in ((0, "qkv"), (2, "o"), (3, "gate_up"), (4, "down")):
        k = 5 * layer + j
        g = int(grid[k])
        if g == 0:
            continue
        prev = st[k - 1, :int(grid[k - 1]), 3].max()
        lines.append(f"{name} (layer {layer}):")
        for cta in range(min(4, g)):
            ev = flat[k, cta * events_per_cta:cta * events_per_cta + 4] - prev
            ch = flat[k, chunk_base + cta * 2 * CHUNKS:chunk_base + (cta + 1) * 2 * CHUNKS].reshape(CHUNKS, 2)
            spans = " ".join(f"{(a - prev) / 1e3:.2f}-{(b - prev) / 1e3:.2f}" for a, b in ch if a > 0)
            lines.append(f"  cta {cta}: entry {ev[0] / 1e3:.2f} wait {ev[2] / 1e3:.2f} ready {ev[1] / 1e3:.2f} "
                         f"exit {ev[3] / 1e3:.2f} | chunks {spans}")
    return "\n".join(lines)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--decode", type=int, default=200)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--chunks", type=int, default=-1, help="layer whose per-chunk stamps to print")
    a = ap.parse_args(argv)
    cfg = dict(LLAMA2_7B, n_layers=a.layers)
    m = Model(cfg)
    m.synthesize(a.seed)
    m.forward(synth_tokens(a.seed, 0, cfg["vocab"], a.prompt), want_logits=False)
    m.decode_steps(a.decode)
    m.status()
    stamps, grid = m.trace_kernels()
    m.close()
    t0 = stamps[0, :grid[0], 0].astype(np.int64).min()
    step = (stamps[5 * a.layers, :grid[5 * a.layers], 3].astype(np.int64).max() - t0) / 1e3
    tab = layer_table(stamps, grid, a.layers)
    print(f"one decode step at position {a.prompt + a.decode}: {step:.1f} us ({a.layers} layers + lm_head)")
    print("per layer, mean over layers 1..L-1, us from the previous kernel's last exit:")
    keys = ("span", "entry_first", "entry_med", "wait_done", "ready", "exit_med", "exit_last")
    print("| kernel | " + " | ".join(keys) + " |")
    print("|---" * (len(keys) + 1) + "|")
    for n in NAMES:
        if n in tab:
            print(f"| {n} | " + " | ".join(f"{tab[n].get(k, float('nan')):.2f}" for k in keys) + " |")
    print(f"| layer | {sum(tab[n]['span'] for n in tab):.2f} | | | | | | |")
    if a.chunks >= 1:
        print(chunk_view(stamps, grid, a.chunks, 4, 160 * 4, cfg["n_kv_heads"]))


if __name__ == "__main__":
    main()
