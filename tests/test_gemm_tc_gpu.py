"""The tcgen05 tensor-core GEMM behind fused_matmul at M > 8 (fp16 scales,
K a multiple of 64) against the oracle's block-quant matmul
(src/fused_matmul.cpp:70-169's intended product, restated).

The GEMM carries the activation as three bf16 parts and the dequantized
weight as two (exact), so the bar is fp32-level: |gpu - oracle| <=
2e-6 * sum_k |x_k w_k| + 1e-6 (both sides round in fp32, in a different
order). Shapes cover the tile sizes (32, 64, 128 activation rows per tile),
ragged M and N, the split-K path (few tiles, long K) and one tile per CTA
(many tiles)."""
import numpy as np
import pytest

import aaedn_b200 as ab
from gpu_util import dev, empty_f32, host

pytestmark = pytest.mark.gpu


def _case(oracle, M, N, K, seed, lda=None, ldc=None, outliers=False):
    data, scales = ab.quantize_q4(ab.synth_normal(seed, 7, N * K))
    lda = lda or K
    ldc = ldc or N
    rng = np.random.default_rng(seed)
    xm = rng.normal(0, 1, (M, lda)).astype(np.float32)
    if outliers:  # one element 10^4 times its 32-block in every block
        blk = xm[:, :K].reshape(M, K // 32, 32)
        pick = rng.integers(0, 32, blk.shape[:2])
        np.put_along_axis(blk, pick[..., None], 1e4, 2)
        xm[:, :K] = blk.reshape(M, K)
    out = empty_f32(M * ldc)
    ab.fused_matmul(dev(xm), dev(data), dev(scales), out, M, N, K, lda=lda, ldc=ldc)
    got = host(out).reshape(M, ldc)[:, :N]
    want = oracle.q4_matmul(np.ascontiguousarray(xm[:, :K]), data, scales, N, K)
    wd = oracle.dequant(data, scales, N * K, f16=True).reshape(N, K)
    bound = 2e-6 * (np.abs(xm[:, :K]) @ np.abs(wd).T) + 1e-6
    err = np.abs(got - want)
    assert np.all(err <= bound), (M, N, K, float(err.max()), float((err / bound).max()))


@pytest.mark.parametrize("M,N,K", [(9, 256, 512), (16, 4096, 4096), (32, 384, 1024), (33, 200, 256),
                                   (64, 4096, 4096), (64, 11008, 4096), (64, 4096, 11008), (100, 1000, 640),
                                   (128, 512, 2048), (200, 256, 512), (2048, 256, 512)])
def test_tc_gemm_vs_oracle(oracle, M, N, K):
    _case(oracle, M, N, K, seed=M + N + K)


def test_tc_gemm_strides_and_outliers(oracle):
    _case(oracle, 40, 300, 512, seed=5, lda=520, ldc=310)
    _case(oracle, 64, 512, 1024, seed=6, outliers=True)


def test_tc_gemm_launches_the_tensor_core_kernel():
    """M > 8 runs the tensor-core path: one split kernel, one GEMM launch and
    (when the tile grid is small) one split-K reduction, not M / 8 GEMVs."""
    M, N, K = 64, 4096, 4096
    data, scales = ab.quantize_q4(ab.synth_normal(1, 2, N * K))
    x = dev(np.ones((M, K), np.float32))
    out = empty_f32(M * N)
    n0 = ab.kernel_launches()
    ab.fused_matmul(x, dev(data), dev(scales), out, M, N, K)
    ab.device_sync()
    assert ab.kernel_launches() - n0 in (2, 3)
