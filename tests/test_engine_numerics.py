"""The arithmetic of the decode GEMV's integer engine (gemv_tiled_i8_kernel),
restated with numpy on the CPU: the activation of each 32-element block is
scaled to y = x * (119 / max|x|) in fp32, each y becomes the integer
Y = rint(y * 2^21) (odd elements: rint(y * 2^17), the high nibble carries a
factor 16). Per code byte (even element in the low nibble, odd in the high)
the tensor-core MMA meets the raw byte lo + 16 hi with the digits of the even
element's Y and the high nibble 16 hi with the digits of Yodd - Yeven, so
that the sum is lo * Yeven + 16 hi * Yodd; both are split into four balanced
base-128 digits, the dot products are exact integers (each MMA covers two
blocks and gives all four digit sums of both), and the digit pairs' sums are
converted to fp32 (rounded to 24 bits), scaled by the lanes that hold them,
digits (0, 1) at weight 1 and digits (2, 3) at 2^-14, then added, as the
kernel does. This pins the engine's precision: the error of an element is
below |w| * max|x of its block| * 1e-7 (the digits keep 2^-21 of the block's
scale, odd elements 2^-17 of y / 16), plus fp32 rounding of the partial sums
and their accumulation; on the normally distributed activations of the GPU
tests that is far inside their bound of 2e-5 * sum|x * w|. No GPU."""
import numpy as np
import pytest


def _digits(Y):
    """Balanced base-128 digits of int64 Y: Y = d0 2^21 + d1 2^14 + d2 2^7 + d3."""
    d0 = (Y + (1 << 20)) >> 21
    r0 = Y - (d0 << 21)
    d1 = (r0 + (1 << 13)) >> 14
    r1 = r0 - (d1 << 14)
    d2 = (r1 + 64) >> 7
    d3 = r1 - (d2 << 7)
    return d0, d1, d2, d3


def engine_dot(codes, scales, x):
    """One output row: codes uint8 [K] (0..15, the weight's nibbles), fp16
    scales [K/32], x fp32 [K]. Mirrors the kernel's roundings."""
    K = x.size
    acc_hi = np.float32(0)  # the lanes holding digits (0, 1)
    acc_lo = np.float32(0)  # the lanes holding digits (2, 3)
    for b in range(K // 32):
        xb = x[32 * b:32 * b + 32].astype(np.float32)
        cb = codes[32 * b:32 * b + 32].astype(np.int64)
        mx = np.float32(np.abs(xb).max())
        inv = np.float32(119.0) / mx if mx > 0 else np.float32(0)
        y = (xb * inv).astype(np.float32)
        mult = np.where(np.arange(32) % 2 == 0, np.float32(2.0 ** 21), np.float32(2.0 ** 17)).astype(np.float32)
        Y = np.rint((y * mult).astype(np.float32)).astype(np.int64)
        ye, yo = Y[0::2], Y[1::2]
        raw = cb[0::2] + 16 * cb[1::2]  # the code byte as the MMA reads it
        hi16 = 16 * cb[1::2]            # its high nibble, masked
        de, dd = _digits(ye), _digits(yo - ye)
        p0, p1, q0, q1 = (int(np.dot(raw, de[k]) + np.dot(hi16, dd[k])) for k in range(4))
        bsc = np.float32(mx / np.float32(119.0 * 128.0))
        sw = np.float32(np.float16(scales[b]).astype(np.float32))
        acc_hi = np.float32(acc_hi + np.float32(sw * bsc) * np.float32(p0 * 128 + p1))
        acc_lo = np.float32(acc_lo + np.float32(sw * np.float32(bsc * np.float32(1.0 / 16384.0))) *
                            np.float32(q0 * 128 + q1))
    return np.float32(acc_hi + acc_lo)


@pytest.mark.parametrize("seed,dist", [(0, "normal"), (1, "wide"), (2, "sparse"), (3, "tiny")])
def test_engine_dot_error_bound(seed, dist):
    rng = np.random.default_rng(seed)
    K = 4096
    for _ in range(8):
        if dist == "normal":
            x = rng.normal(0, 1, K)
        elif dist == "wide":  # magnitudes over 12 orders inside and across blocks
            x = rng.normal(0, 1, K) * 10.0 ** rng.uniform(-6, 6, K)
        elif dist == "sparse":
            x = rng.normal(0, 1, K) * (rng.random(K) < 0.05)
        else:
            x = rng.normal(0, 1e-30, K)
        x = x.astype(np.float32)
        codes = rng.integers(0, 16, K).astype(np.uint8)
        scales = rng.uniform(1e-3, 1e-1, K // 32).astype(np.float16)
        w = codes.astype(np.float64) * np.repeat(scales.astype(np.float64), 32)
        x64 = x.astype(np.float64)
        exact = float(np.dot(w, x64))
        got = float(engine_dot(codes, scales, x))
        mag = float(np.dot(np.abs(w), np.abs(x64)))
        blockmax = np.repeat(np.abs(x64).reshape(-1, 32).max(1), 32)
        quant = float(np.dot(np.abs(w), blockmax)) * 1e-7
        assert abs(got - exact) <= quant + 1e-6 * mag + 1e-37, (got, exact, quant, mag)
        if dist == "normal":
            assert abs(got - exact) <= 2e-6 * mag  # ten times inside the GPU tests' bound


def test_digits_are_balanced_and_exact():
    """Digits of Yeven (|y| <= 119) and of Yodd - Yeven (up to 119 * 17 / 16
    times 2^21) fit signed bytes, and the digit sums the kernel forms
    (c0 * 128 + c1 over a block's 16 bytes) stay inside int32."""
    rng = np.random.default_rng(9)
    lim = (119 << 21) + (119 << 17)
    Y = np.concatenate([rng.integers(-lim, lim + 1, 100000), [lim, -lim, 119 << 21, -(119 << 21)]]).astype(np.int64)
    d0, d1, d2, d3 = _digits(Y)
    assert np.array_equal(d0 * (1 << 21) + d1 * (1 << 14) + d2 * (1 << 7) + d3, Y)
    assert np.abs(d0).max() <= 127 and max(np.abs(d).max() for d in (d1, d2, d3)) <= 64
    c0 = 16 * 255 * 119 + 16 * 240 * 127
    c1 = 16 * 255 * 64 + 16 * 240 * 64
    assert c0 * 128 + c1 < 2 ** 31
