"""Batched sequences over a shared, paged KV cache (aaedn_model_create_batched)
against the oracle, which runs every sequence on its own.

The reference keeps one segment table per agent (src/kvcache.cpp:15-60) and
describes branches that continue from a parent's tokens and are pruned
(docs/sdd.md:206-215, src/agent.cpp:107-140); here a sequence is a page
table in device memory, a fork shares the parent's pages and copies a shared
page before either side appends into it, and closing a sequence releases the
pages nobody else holds. Checked:
  * several sequences with different prompts and lengths stepped together
    give each sequence's own greedy tokens and logits;
  * a prompt forked into four branches (the 70B workload's shape, at small
    widths) that continue with different tokens: each branch equals the
    oracle run of prompt + its own continuation, and the parent is unchanged
    by its children's appends (the shared tail page was copied);
  * closing returns exactly the pages no other sequence holds.
Bars as the model tests: tokens identical, logits within 1e-4 relative."""
import numpy as np
import pytest

import aaedn_b200 as ab
import pyoracle

pytestmark = pytest.mark.gpu

GQA = dict(dim=256, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=32, ffn_dim=512, vocab=1000, max_seq=256,
           rope_theta=500000.0, eps=1e-6)


def _rel_err(a, b):
    return float(np.abs(a - b).max() / max(1e-30, np.abs(b).max()))


def _oracle_run(om, tokens):
    om.reset()
    lg = None
    for t in tokens:
        lg = om.step(int(t))
    return lg


@pytest.fixture(scope="module")
def pair():
    w = ab.synthetic_weights(GQA, 5)
    om = pyoracle.OracleModel(pyoracle.Oracle(), GQA, w)
    bm = ab.BatchedModel(GQA, max_seqs=8, kv_tokens=8 * 256)
    bm.set_weights(w)
    yield w, om, bm
    bm.close()


def test_sequences_stepped_together_match_each_alone(pair):
    w, om, bm = pair
    lens = [5, 33, 64, 70, 2, 17]  # page boundaries (64 tokens) on both sides; more than 4 rows: the tiled lm_head
    seqs, hist = [], []
    for i, n in enumerate(lens):
        s = bm.open()
        p = ab.synth_tokens(5, 10 + i, GQA["vocab"], n)
        _, nxt = bm.prefill(s, p)
        seqs.append(s)
        hist.append(list(p) + [nxt])
    for step in range(24):
        toks = [h[-1] for h in hist]
        logits, nxt = bm.step(seqs, toks)
        for i, h in enumerate(hist):
            want = _oracle_run(om, h)
            assert _rel_err(logits[i], want) < 1e-4, (step, i)
            assert int(nxt[i]) == int(np.argmax(want)), (step, i)
            h.append(int(nxt[i]))
    for s, h in zip(seqs, hist):
        assert bm.seq_len(s) == len(h) - 1
        bm.close_seq(s)
    total, free = bm.kv_pages()
    assert free == total


def test_fork_four_branches_copy_on_write(pair):
    w, om, bm = pair
    total, free0 = bm.kv_pages()
    root = bm.open()
    prompt = ab.synth_tokens(5, 99, GQA["vocab"], 100)  # 1 full page + a shared partial page
    _, first = bm.prefill(root, prompt)
    kids = [bm.fork(root) for _ in range(4)]
    # forks share every page: no page allocated yet
    assert bm.kv_pages()[1] == free0 - 2
    cont = {k: [int((first + 7 * j) % GQA["vocab"])] for j, k in enumerate(kids)}
    for step in range(12):
        logits, nxt = bm.step(kids, [cont[k][-1] for k in kids])
        for i, k in enumerate(kids):
            want = _oracle_run(om, list(prompt) + cont[k])
            assert _rel_err(logits[i], want) < 1e-4, (step, i)
            cont[k].append(int(nxt[i]))
    # each branch copied the shared tail page once; the root still decodes
    # as if the branches never existed
    lg, nxt = bm.prefill(root, [first])
    want = _oracle_run(om, list(prompt) + [first])
    assert _rel_err(lg, want) < 1e-4 and nxt == int(np.argmax(want))
    used = free0 - bm.kv_pages()[1]
    assert used == 2 + 4  # root's two pages + one copied tail page per branch
    for k in kids:
        bm.close_seq(k)
    assert bm.kv_pages()[1] == free0 - 2  # the root's pages stay
    bm.close_seq(root)
    assert bm.kv_pages()[1] == free0


def test_batched_rejects_what_it_cannot_do(pair):
    w, om, bm = pair
    s = bm.open()
    with pytest.raises(ab.AaednError):
        bm.step([s, s], [1, 2])  # one sequence twice in a batch
    with pytest.raises(ab.AaednError):
        bm.forward([1, 2, 3])  # the single-sequence calls
    bm.close_seq(s)
    with pytest.raises(ab.AaednError):
        bm.step([s], [1])  # closed


def test_batched_at_8b_widths_splits_the_paired_epilogues():
    """Three sequences of the Llama-3-8B widths (2 layers, GQA 32/8, ffn
    14336, vocab 128256) prefilled and stepped together: at so few rows the
    qkv and gate/up GEMMs split K across CTAs, and the RoPE / K,V-append and
    SwiGLU epilogues run in the split-K reduction. Each sequence's logits
    and tokens match the oracle's run of that sequence alone."""
    cfg = dict(ab.LLAMA3_8B, n_layers=2, max_seq=128)
    w = ab.synthetic_weights(cfg, 909)
    om = pyoracle.OracleModel(pyoracle.Oracle(), cfg, w)
    bm = ab.BatchedModel(cfg, max_seqs=4, kv_tokens=4 * 128)
    try:
        bm.set_weights(w)
        seqs, hist = [], []
        for i, n in enumerate((3, 6, 9)):
            s = bm.open()
            p = ab.synth_tokens(909, i, cfg["vocab"], n)
            _, nxt = bm.prefill(s, p)
            seqs.append(s)
            hist.append(list(p) + [nxt])
        for _ in range(3):
            logits, nxt = bm.step(seqs, [h[-1] for h in hist])
            for i, h in enumerate(hist):
                h.append(int(nxt[i]))
        for i, h in enumerate(hist):
            want = _oracle_run(om, h[:-1])
            assert _rel_err(logits[i], want) < 1e-4, i
            assert h[-1] == int(np.argmax(want)), i
    finally:
        bm.close()
