"""The exact split of an fp32 activation into bf16 terms that the tensor-core
GEMMs take (k_pf_split, and the row kernels of the batched decode):

    hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid)

(round to nearest even; each difference exact in fp32).  Restated here with
numpy on the host: three terms carry every bit of a normal fp32 value, two
terms carry x to 2^-17 of |x|.  Every weight of a bf16 codebook is exact in
bf16, so each product term * w is exact in fp32 and the GEMM's only error is
its accumulation order."""
import numpy as np


def _bf16_rne(v: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32."""
    u = v.astype(np.float32).view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    return (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def _split(x: np.ndarray, terms: int):
    out, r = [], x.astype(np.float32)
    for _ in range(terms):
        b = _bf16_rne(r)
        out.append(b)
        r = (r - b).astype(np.float32)   # exact: b holds r's leading bits
    return out


def _values(seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(200000).astype(np.float32)
    scales = np.float32(2.0) ** rng.integers(-100, 100, x.size).astype(np.float32)
    return np.concatenate([x, (x * scales).astype(np.float32),
                           np.array([1.0, -1.0, 3.0e38, -1.5e-30, 65504.0, 1 / 3],
                                    np.float32)])


def test_three_terms_are_exact():
    x = _values(1)
    hi, mid, lo = _split(x, 3)
    # the sum in float64 (exact for three bf16 numbers of these exponents)
    back = hi.astype(np.float64) + mid.astype(np.float64) + lo.astype(np.float64)
    np.testing.assert_array_equal(back, x.astype(np.float64))


def test_two_terms_within_2_pow_minus_17():
    x = _values(2)
    hi, mid = _split(x, 2)
    back = hi.astype(np.float64) + mid.astype(np.float64)
    rel = np.abs(back - x.astype(np.float64)) / np.abs(x.astype(np.float64))
    assert rel.max() <= 2.0 ** -17


def test_bf16_rounding_is_nearest_even():
    # 1 + 2^-8 lies halfway between the bf16 neighbours 1 and 1 + 2^-7: even -> 1
    x = np.array([1 + 2 ** -8, 1 + 3 * 2 ** -8, 1 + 2 ** -9], np.float32)
    np.testing.assert_array_equal(_bf16_rne(x),
                                  np.array([1.0, 1 + 2 ** -6, 1.0], np.float32))
