"""The sampling restatement (oracle/pyoracle.py sample_ref, the reference's
spec of docs/mpd.md:539-554) pinned against src/main.cpp's own softmax draw
(sample_main_ref): at temperature 1 and top_p 1 both realise the same
distribution. No GPU."""
import numpy as np

import pyoracle


def test_sorted_draw_has_the_reference_distribution():
    rng = np.random.default_rng(11)
    V, n = 16, 4096
    lg = rng.normal(0, 1.5, V).astype(np.float32)
    us = (np.arange(n) + 0.5) / n
    a = np.bincount([pyoracle.sample_ref(lg, 1.0, 1.0, u)[0] for u in us], minlength=V)
    b = np.bincount([pyoracle.sample_main_ref(lg, u) for u in us], minlength=V)
    assert np.abs(a - b).max() <= 2


def test_greedy_and_narrow_nucleus_pick_the_argmax():
    rng = np.random.default_rng(5)
    lg = rng.normal(0, 2, 500).astype(np.float32)
    top = int(np.argmax(lg))
    assert pyoracle.sample_ref(lg, 0.0, 0.9, 0.7)[0] == top
    assert pyoracle.sample_ref(lg, 1.0, 1e-9, 0.999)[0] == top


def test_nucleus_keeps_only_the_top_mass():
    # p = (0.5, 0.3, 0.2) at T = 1: top_p 0.6 keeps ids 0 and 1 (0.8 of the mass)
    lg = np.log(np.array([0.5, 0.3, 0.2], np.float32))
    picks = {pyoracle.sample_ref(lg, 1.0, 0.6, u)[0] for u in np.linspace(0, 0.999, 200)}
    assert picks == {0, 1}
    assert pyoracle.sample_ref(lg, 1.0, 0.6, 0.6)[0] == 0   # 0.6 * 0.8 = 0.48 < 0.5
    assert pyoracle.sample_ref(lg, 1.0, 0.6, 0.7)[0] == 1   # 0.56 > 0.5
