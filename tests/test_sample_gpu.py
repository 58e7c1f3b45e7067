"""aaedn_cu_sample (temperature, top-p, multinomial draw on the device)
against the sorted restatement of the reference's sampling spec
(docs/mpd.md:539-554) and against the distribution of src/main.cpp's own
softmax draw.

Token choices are index work and must match exactly, except where the
restatement reports a decision closer than 1e-5 relative to a threshold
(fp32 exp on the host and the device may differ by an ulp there)."""
import numpy as np
import pytest

import aaedn_b200 as ab
import pyoracle
from gpu_util import dev, host

pytestmark = pytest.mark.gpu


def _tokens(n):
    import torch
    return torch.full((n,), 0xFFFFFFF, dtype=torch.int32, device="cuda")


def _sample_many(logits, temperature, top_p, us):
    d_l = dev(np.asarray(logits, np.float32))
    out = _tokens(len(us))
    for k, u in enumerate(us):
        ab.sample(d_l, len(logits), temperature, top_p, u, out[k:k + 1])
    return host(out).astype(np.int64)


def test_greedy_is_argmax_with_ties_to_the_lowest_id():
    rng = np.random.default_rng(3)
    for V in (1, 5, 1000, 32000):
        lg = rng.normal(0, 2, V).astype(np.float32)
        if V > 10:
            lg[V // 3] = lg[V - 2] = lg.max() + 1.0  # a tie: the lower id wins
        got = _sample_many(lg, 0.0, 0.9, [0.5, 0.0])
        assert (got == int(np.argmax(lg))).all()


@pytest.mark.parametrize("V", [7, 1000, 32000])
@pytest.mark.parametrize("temperature", [0.5, 0.8, 1.0, 1.7])
@pytest.mark.parametrize("top_p", [0.1, 0.9, 0.95, 1.0])
def test_matches_sorted_restatement(V, temperature, top_p):
    rng = np.random.default_rng(V * 7 + int(temperature * 10) + int(top_p * 100))
    lg = rng.normal(0, 2.5, V).astype(np.float32)
    lg[rng.integers(0, V, 3)] = lg.max()  # equal probabilities: ordered by id
    us = np.concatenate([[0.0, 0.999999], rng.random(10)]).astype(np.float32)
    got = _sample_many(lg, temperature, top_p, us)
    for u, g in zip(us, got):
        want, margin = pyoracle.sample_ref(lg, temperature, top_p, float(u))
        assert g == want or margin < 1e-5, (u, g, want, margin)


def test_same_distribution_as_the_reference_draw():
    """T = 1, top_p = 1: over a regular grid of u the device's sorted-order
    draw and src/main.cpp's id-order draw pick every token the same number
    of times, up to the grid's resolution."""
    rng = np.random.default_rng(11)
    V, n = 16, 4096
    lg = rng.normal(0, 1.5, V).astype(np.float32)
    us = ((np.arange(n) + 0.5) / n).astype(np.float32)
    got = _sample_many(lg, 1.0, 1.0, us)
    ref = np.array([pyoracle.sample_main_ref(lg, float(u)) for u in us])
    cg = np.bincount(got, minlength=V)
    cr = np.bincount(ref, minlength=V)
    assert np.abs(cg - cr).max() <= 2, (cg, cr)


def test_rejects_bad_arguments():
    d_l = dev(np.zeros(8, np.float32))
    out = _tokens(1)
    for t, p, u in ((1.0, 0.0, 0.5), (1.0, 1.5, 0.5), (1.0, 0.9, 1.0), (1.0, 0.9, -0.1)):
        with pytest.raises(ab.AaednError):
            ab.sample(d_l, 8, t, p, u, out)
    with pytest.raises(ab.AaednError):
        ab.sample(np.zeros(8, np.float32), 8, 1.0, 0.9, 0.5, out)  # host logits
