"""The arithmetic facts the tensor-core projections rest on (ovf_tc.cu,
ovf_tc6.cu, ovf_tc8.cu), checked exhaustively on the host: every fp16
operand and offset they form is exactly representable, the magic-number
expansion (0x6400 | q = 1024 + q, one fused multiply-add by a scale) yields
the exact integer product, and every fp32 accumulator's partial sums stay
below 2^24 in magnitude, so the tensor cores' sums are exact in any order.
With these, the kernels reproduce the reference's integer dot products
(Runtime/Q4KDotKernel.cs:216-256, Runtime/Q6KDotKernel.cs:77-225,
Runtime/Q8DotKernel.cs:99-140) exactly, and the fp32 tails they run in the
epilogue are the reference's own operations."""
import numpy as np

F16_EXACT_INT = 2048      # every integer of magnitude <= 2048 is an fp16
FP32_EXACT_INT = 1 << 24  # every integer of magnitude <= 2^24 is an fp32
Q8_MAX = 128              # |Q8_K / Q8_0 activation quant| (the quantizers clamp to 127)


def f16_exact(v) -> bool:
    v = np.asarray(v, dtype=np.float64)
    return bool(np.all(np.float16(v).astype(np.float64) == v))


def fma_f16(x, s, off):
    """fp16 fma: the exact x * s + off rounded once to fp16."""
    return np.float16(np.asarray(x, np.float64) * np.asarray(s, np.float64) + np.asarray(off, np.float64))


def test_magic_number_expansion_is_exact_for_q4k():
    q = np.arange(16)                       # 4-bit values
    sc = np.arange(64)                      # 6-bit scales
    x = np.float16(1024 + q)                # 0x6400 | q
    assert f16_exact(1024 + q)
    assert f16_exact(-1024 * sc)            # the offset of every scale
    got = fma_f16(x[:, None], sc[None, :], -1024.0 * sc[None, :])
    want = q[:, None] * sc[None, :]         # 0 .. 945
    assert np.all(got.astype(np.float64) == want) and want.max() <= F16_EXACT_INT


def test_magic_number_expansion_is_exact_for_q6k_split_scales():
    q = np.arange(64)                       # 6-bit values
    sc = np.arange(-128, 128)               # signed 8-bit sub-block scales
    sl, sh = sc & 15, sc >> 4               # sc = 16 sh + sl
    assert np.all(16 * sh + sl == sc) and sl.min() == 0 and sl.max() == 15 and sh.min() == -8 and sh.max() == 7
    x = np.float16(1024 + q)
    for s in (sl, sh):
        assert f16_exact(-1056 * s)         # 1056 s = 33 s * 32: at most 11 significant bits
        got = fma_f16(x[:, None], s[None, :], -1056.0 * s[None, :])
        want = (q[:, None] - 32) * s[None, :]
        assert np.all(got.astype(np.float64) == want) and np.abs(want).max() <= F16_EXACT_INT
    # the recombination lo + 16 hi is the reference's per-element product
    lo = (q[:, None] - 32) * sl[None, :]
    hi = (q[:, None] - 32) * sh[None, :]
    assert np.all(lo + 16 * hi == (q[:, None] - 32) * sc[None, :])


def test_activation_quants_and_bsums_are_exact_fp16():
    assert f16_exact(np.arange(-Q8_MAX, Q8_MAX + 1))           # Q8_K quants as fp16
    assert f16_exact(np.arange(-16 * Q8_MAX, 16 * Q8_MAX + 1))  # 16-element bsums (Q4_K minAcc MMA)


def test_accumulators_stay_below_2_24():
    # Q4_K main accumulators: one per K half of a super-block (128 products of q4*sc x q8)
    assert 128 * (15 * 63) * Q8_MAX < FP32_EXACT_INT
    # Q4_K minAcc: 16 products of m (6-bit) x bsum16
    assert 16 * 63 * (16 * Q8_MAX) < FP32_EXACT_INT
    # Q6_K lo / hi accumulators: 256 products per super-block
    assert 256 * (32 * 15) * Q8_MAX < FP32_EXACT_INT
    assert 256 * (32 * 8) * Q8_MAX < FP32_EXACT_INT
    # the int32 recombinations cannot overflow
    assert 2 * 128 * 945 * Q8_MAX + 8 * 16 * 63 * 16 * Q8_MAX < 2 ** 31          # Q4_K mainAcc
    assert 256 * 32 * 128 * Q8_MAX < 2 ** 31                                      # Q6_K mainAcc
    # Q8_0: one int8 x int8 block of 32 in an int32 accumulator
    assert 32 * 127 * Q8_MAX < 2 ** 31


def test_fp32_add_of_two_exact_halves_is_the_rounded_integer():
    """(float)mainAcc == fadd(lo, hi) when lo and hi are exact integers: the
    add rounds the exact sum once, as the int -> float conversion does."""
    rng = np.random.default_rng(0)
    lim = 128 * 945 * Q8_MAX
    lo = rng.integers(-lim, lim + 1, 200000)
    hi = rng.integers(-lim, lim + 1, 200000)
    fadd = (lo.astype(np.float32) + hi.astype(np.float32)).astype(np.float32)
    assert np.all(lo.astype(np.float32).astype(np.int64) == lo)
    assert np.all(fadd == (lo + hi).astype(np.float32))
