"""fused_matmul on weights repacked into the model's tile-major layout
(aaedn_q4_repack_tiled + aaedn_cu_fused_matmul_tiled) against the oracle's
block-quant matmul (src/fused_matmul.cpp:70-169's intended product).

M == 1 runs the decode GEMV engine (integer MMA over the activation's
base-128 digits: |err| <= 2e-5 * sum|x w| + 1e-6, the GEMV bound of the
kernel tests), M > 1 the tcgen05 GEMM (2e-6 * sum|x w| + 1e-6). The repack
itself is checked by the products: a misplaced code or scale changes them
far beyond either bound."""
import numpy as np
import pytest

import aaedn_b200 as ab
from gpu_util import dev, empty_f32, host

pytestmark = pytest.mark.gpu


def _case(oracle, M, N, K, seed, outliers=False):
    data, scales = ab.quantize_q4(ab.synth_normal(seed, 9, N * K))
    tiled = ab.repack_tiled(data, scales, N, K)
    rng = np.random.default_rng(seed)
    xm = rng.normal(0, 1, (M, K)).astype(np.float32)
    if outliers:  # one element 10^4 times its 32-block, and mostly-zero blocks
        blk = xm.reshape(M, K // 32, 32)
        pick = rng.integers(0, 32, blk.shape[:2])
        np.put_along_axis(blk, pick[..., None], 1e4, 2)
        blk[:, ::3, 1:] = 0.0
        xm = blk.reshape(M, K)
    out = empty_f32(M * N)
    ab.fused_matmul_tiled(dev(xm), dev(tiled), out, M, N, K)
    got = host(out).reshape(M, N)
    want = oracle.q4_matmul(xm, data, scales, N, K)
    wd = oracle.dequant(data, scales, N * K, f16=True).reshape(N, K)
    rel = 2e-5 if M == 1 else 2e-6
    bound = rel * (np.abs(xm) @ np.abs(wd).T) + 1e-6
    err = np.abs(got - want)
    assert np.all(err <= bound), (M, N, K, float(err.max()), float((err / bound).max()))


@pytest.mark.parametrize("M,N,K", [(1, 512, 1024), (1, 4096, 4096), (1, 4096, 11008), (8, 512, 1024),
                                   (8, 11008, 4096), (64, 4096, 4096), (64, 4096, 11008), (37, 272, 640)])
def test_tiled_matmul_vs_oracle(oracle, M, N, K):
    _case(oracle, M, N, K, seed=M + N + K)


def test_tiled_matmul_outliers(oracle):
    _case(oracle, 1, 1024, 2048, seed=3, outliers=True)
    _case(oracle, 16, 1024, 2048, seed=4, outliers=True)


def test_tiled_matmul_rejects_shapes_it_does_not_tile():
    data, scales = ab.quantize_q4(ab.synth_normal(1, 1, 24 * 256))
    with pytest.raises(ab.AaednError):
        ab.repack_tiled(data, scales, 24, 256)  # N not a multiple of 16
    out = empty_f32(64)
    with pytest.raises(ab.AaednError):
        ab.fused_matmul_tiled(out, out, out, 1, 16, 96)  # K not a multiple of 128
