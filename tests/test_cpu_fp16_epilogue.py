"""The GEMM epilogue's packed-fp16 form (tc_gemm.cu, epilogue8 with no
activation or ReLU) replaces the reference's fp32 formula
`half(float(round_half(acc)) + float(bias))` (and the same again for the
residual) by fp16 additions. The two agree bit for bit iff rounding the fp32
sum of two fp16 values to fp16 equals rounding their exact sum. This checks
that claim on every finite fp16 value against a set of partners that covers
every exponent distance, carries and borrows at the binade edges, and
subnormals; exact sums are formed in float64 (two fp16 values always sum
exactly in 53 bits). An exhaustive run over all pairs of finite fp16 values
found no mismatch either; it takes minutes, this subset seconds."""

import numpy as np


def _finite_fp16() -> np.ndarray:
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    return h[np.isfinite(h)]


def _partners(rng) -> np.ndarray:
    f = _finite_fp16()
    mant = np.arange(1024, dtype=np.uint16)
    picks = [f[rng.integers(0, f.size, 2048)]]
    # every exponent, smallest / largest / random mantissas, both signs
    for e in range(31):
        for m in (mant[:4], mant[-4:], rng.choice(mant, 8)):
            bits = (np.uint16(e) << np.uint16(10)) | m
            picks.append(bits.astype(np.uint16).view(np.float16))
            picks.append((bits | np.uint16(0x8000)).astype(np.uint16).view(np.float16))
    return np.concatenate(picks)


def test_fp16_sum_rounding_equals_fp32_path():
    rng = np.random.default_rng(7)
    a = _finite_fp16()
    b = _partners(rng)
    a32, a64 = a.astype(np.float32), a.astype(np.float64)
    with np.errstate(over="ignore"):
        for bv in b:
            via32 = (a32 + np.float32(bv)).astype(np.float16)
            exact = (a64 + np.float64(bv)).astype(np.float16)
            diff = via32.view(np.uint16) != exact.view(np.uint16)
            diff &= ~((via32 == 0) & (exact == 0))  # +0 / -0
            assert not diff.any(), (bv, a[np.nonzero(diff)[0][:4]])


def test_relu_commutes_with_rounding():
    x = np.random.default_rng(8).standard_normal(1 << 16).astype(np.float32) * 100
    assert np.array_equal(np.maximum(x, 0).astype(np.float16), np.maximum(x.astype(np.float16), np.float16(0)))
