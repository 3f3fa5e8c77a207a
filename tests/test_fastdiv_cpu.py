"""The GEMM scheduler's FastDiv (gemm_core.cuh): a / d as trunc(float(a) *
float(1/d)) plus one correction step, claimed exact for 0 <= a < 2^24. The
float32 arithmetic is emulated with numpy (round-to-nearest products,
truncating conversion, as on the device)."""
import numpy as np
import pytest


def fastdiv(a: np.ndarray, d: int) -> np.ndarray:
    r = np.float32(1.0) / np.float32(d)
    q = (a.astype(np.float32) * r).astype(np.int64)  # float product, truncation
    rem = a - q * d
    q = np.where(rem < 0, q - 1, q)
    q = np.where(rem >= d, q + 1, q)
    return q


@pytest.mark.parametrize("d", [1, 2, 3, 7, 16, 37, 64, 127, 148, 255, 1000, 4099, 65521,
                               1 << 20, (1 << 24) - 3])
def test_fastdiv_is_exact_below_2_pow_24(d):
    rng = np.random.default_rng(d)
    a = np.concatenate([np.arange(0, 70000), rng.integers(0, 1 << 24, 200000),
                        (1 << 24) - 1 - np.arange(1000)]).astype(np.int64)
    # multiples of d and their neighbours are where a truncated estimate goes wrong
    m = np.arange(0, (1 << 24) // d + 1, max(1, ((1 << 24) // d) // 50000)) * d
    a = np.concatenate([a, m, m - 1, m + 1])
    a = a[(a >= 0) & (a < (1 << 24))]
    assert np.array_equal(fastdiv(a, d), a // d)
