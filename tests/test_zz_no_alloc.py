"""aaedn_cu_attention_noalloc against aaedn_cu_attention and the oracle.

The no-allocation variant serves callers that may not allocate device memory
after startup (they hand all of it to one fixed pool). It takes its split
partials and counters from one fixed device array that every call shares, so
the checks run it twice in a row, with different inputs and shapes each
time: the second call must not see what the first call left in the array.
Each result is compared with the allocating entry point and with the oracle
(the CPU restatement of src/attention.cpp:10-84 with the head index). With
two GPUs the same calls run on device 0 and then device 1 (the array, its
address and the kernels' shared-memory attribute are per device).
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
    return q, kc, vc, segs


def _check_twice(first, second, oracle):
    for i, (H, hd, T) in enumerate((first, second)):
        q, kc, vc, segs = _case(H, hd, T, seed=100 * i + H * T)
        dq, dk, dv = dev(q), dev(kc), dev(vc)
        scale = 1.0 / np.sqrt(hd)
        want = empty_f32(H * hd)
        ab.attention(dq, dk, dv, segs, want, H, hd, scale)
        got = empty_f32(H * hd)
        ab.attention_noalloc(dq, dk, dv, segs, got, H, hd, scale)
        g = host(got)
        np.testing.assert_allclose(g, host(want), rtol=2e-5, atol=2e-6)
        np.testing.assert_allclose(g, oracle.attention(q, kc, vc, segs.reshape(-1), H, hd, np.float32(scale)),
                                   rtol=2e-5, atol=2e-6)


@pytest.mark.parametrize("first,second", [((32, 128, 640), (32, 128, 640)), ((4, 128, 1000), (2, 64, 5000)),
                                          ((6, 48, 37), (32, 128, 3000))])
def test_noalloc_matches_attention_twice_in_a_row(first, second, oracle):
    _check_twice(first, second, oracle)


def test_noalloc_on_a_second_device(oracle):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    prev = torch.cuda.current_device()
    try:
        for d in (0, 1):
            torch.cuda.set_device(d)
            _check_twice((32, 128, 700), (4, 64, 3000), oracle)
    finally:
        torch.cuda.set_device(prev)


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
