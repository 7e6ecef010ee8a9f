"""Integer-to-float identities that the exact GEMM kernels rely on, checked exhaustively on the CPU.

The block dot products of the Q8 / Q4 formats produce int32 lane sums L (8 int8 x int8 products:
|L| <= 8 * 128 * 128). The kernels convert them without the int-to-float instruction: they add L to
the bit pattern 0x4B400000 (1.5 * 2^23 as fp32; `dp4a` accumulates straight onto it) and subtract
1.5 * 2^23 in fp32 (csrc/common.cuh `lane_sum_f32`, csrc/matmul.cuh `k_gemm4`). That is exact for
|L| < 2^22, because fp32 values in [2^23, 2^24) are spaced exactly 1 apart. These tests check the
claim for every L in that range, and that the largest lane sum of each format lies well inside it.
"""
import numpy as np

BIAS_BITS = 0x4B400000
BIAS = np.float32(12582912.0)  # 1.5 * 2^23


def test_bias_conversion_is_exact_over_the_whole_range():
    lim = 1 << 22
    lane = np.arange(-lim + 1, lim, dtype=np.int64)
    via_bias = (lane + BIAS_BITS).astype(np.int32).view(np.float32) - BIAS
    assert via_bias.dtype == np.float32
    assert np.array_equal(via_bias, lane.astype(np.float32))
    # and the bit patterns, so that -0.0 / +0.0 cannot hide a difference
    assert np.array_equal(via_bias.view(np.uint32), lane.astype(np.float32).view(np.uint32))


def test_block_lane_sums_fit_the_exact_range():
    # Q8 x Q8: 8 products of int8 values (the quantizer emits [-127, 127]; -128 is allowed here)
    q8 = 8 * 128 * 128
    # Q8 activations x Q4 weights (4-bit values stored with an offset of 8: [-8, 7])
    q4 = 8 * 128 * 8
    assert max(q8, q4) < (1 << 22)
    lane = np.array([-q8, -q4, 0, q4, q8], np.int64)
    via_bias = (lane + BIAS_BITS).astype(np.int32).view(np.float32) - BIAS
    assert np.array_equal(via_bias, lane.astype(np.float32))


def test_fp16_products_are_exact_in_fp32():
    """The exact fp16 GEMM (csrc/matmul.cuh `k_gemm_f16`) adds each fp16 x fp16 product into the
    reference's fp32 lane chain with one fused multiply-add. That equals the reference's separate
    multiply and add because the product of two fp16 values (11-bit significands, exponents
    -24..15) is exact in fp32: fma(a, b, c) = RN(a*b + c) = RN(fl(a*b) + c) when fl(a*b) == a*b."""
    # every pair of significands (hidden bit included) at exponent 0 ...
    sig = (1024 + np.arange(1024, dtype=np.float64)) / 1024.0
    a, b = np.meshgrid(sig, sig)
    exact = a * b  # float64 holds the 22-bit product exactly
    assert np.array_equal((a.astype(np.float32) * b.astype(np.float32)).astype(np.float64), exact)
    # ... and pairs drawn from every finite fp16 value, subnormals and the extremes included
    rng = np.random.default_rng(16)
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    vals = bits.view(np.float16)
    vals = vals[np.isfinite(vals)]
    x = rng.choice(vals, 2_000_000).astype(np.float64)
    y = rng.choice(vals, 2_000_000).astype(np.float64)
    x = np.concatenate([x, vals.astype(np.float64)])
    y = np.concatenate([y, np.full(vals.size, 65504.0)])  # the largest magnitude against all
    exact = x * y
    assert np.array_equal((x.astype(np.float32) * y.astype(np.float32)).astype(np.float64), exact)
