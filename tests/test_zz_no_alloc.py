"""aaedn_cu_attention_noalloc against aaedn_cu_attention.

The no-allocation variant serves callers that may not allocate device memory
after startup (they hand all of it to one fixed pool). It takes its split
partials and counters from one fixed device array that every call shares, so
the checks run it twice in a row, with different inputs and shapes each
time: the second call must not see what the first call left in the array.
This file is collected last so that a run stopping at the first failure has
run every other test before it."""
import numpy as np
import pytest

import aaedn_b200 as ab
from gpu_util import dev, empty_f32, host

pytestmark = pytest.mark.gpu


def _case(H, hd, T, seed):
    rng = np.random.default_rng(seed)
    q = rng.normal(0, 1, H * hd).astype(np.float32)
    kc = rng.normal(0, 1, T * H * hd).astype(np.float32)
    vc = rng.normal(0, 1, T * H * hd).astype(np.float32)
    cut = [0, T // 5, T // 2, T]
    segs = np.array([[cut[1], cut[2] - cut[1]], [0, cut[1]], [cut[2], T - cut[2]]], np.uint32)
    return dev(q), dev(kc), dev(vc), segs


@pytest.mark.parametrize("first,second", [((32, 128, 640), (32, 128, 640)), ((4, 128, 1000), (2, 64, 5000)),
                                          ((6, 48, 37), (32, 128, 3000))])
def test_noalloc_matches_attention_twice_in_a_row(first, second):
    for i, (H, hd, T) in enumerate((first, second)):
        q, kc, vc, segs = _case(H, hd, T, seed=100 * i + H * T)
        scale = 1.0 / np.sqrt(hd)
        want = empty_f32(H * hd)
        ab.attention(q, kc, vc, segs, want, H, hd, scale)
        got = empty_f32(H * hd)
        ab.attention_noalloc(q, kc, vc, segs, got, H, hd, scale)
        np.testing.assert_allclose(host(got), host(want), rtol=2e-5, atol=2e-6)


def test_noalloc_rejects_shapes_beyond_the_scratch():
    H, hd = 2048, 128  # 2048 split counters do not fit; rejected before any launch
    q = dev(np.zeros(H * hd, np.float32))
    out = empty_f32(H * hd)
    with pytest.raises(ab.AaednError) as e:
        ab.attention_noalloc(q, q, q, np.array([[0, 1]], np.uint32), out, H, hd, 0.1)
    assert e.value.rc == -1 and "scratch" in str(e.value)


def test_noalloc_empty_segments_give_zeros():
    out = empty_f32(128)
    q = dev(np.ones(128, np.float32))
    ab.attention_noalloc(q, q, q, np.zeros((1, 2), np.uint32), out, 1, 128, 0.1)
    assert np.all(host(out) == 0)
