"""The multiply-high division the GEMM kernel uses for its per-tile index
arithmetic (FastDiv in tosa_b200/csrc/tc_gemm.cuh, make_fastdiv in
gemm_launch.cuh): n / d == (mulhi32(n, m) + n) >> s for 0 <= n < 2^31, with
s = ceil(log2 d) and m = floor(2^32 (2^s - d) / d) + 1, checked here in exact
integer arithmetic with the device's 32-bit wrap."""

import numpy as np
import pytest


def make_fastdiv(d):
    s = 0
    while (1 << s) < d:
        s += 1
    m = ((1 << 32) * ((1 << s) - d)) // d + 1
    assert 0 <= m < (1 << 32)
    return m, s


def fdiv(n, m, s):
    hi = (n * m) >> 32
    return ((hi + n) & 0xFFFFFFFF) >> s


@pytest.mark.parametrize("d", list(range(1, 300)) + [3136, 12544, 50176, 784, 196, 49, 1568, 6272, 65535,
                                                     (1 << 20) + 7, (1 << 30) - 1, 1 << 30])
def test_fastdiv_matches_integer_division(d):
    m, s = make_fastdiv(d)
    rng = np.random.default_rng(d)
    ns = [0, 1, d - 1, d, d + 1, 2 * d - 1, (1 << 31) - 1, (1 << 31) - d] + [int(v) for v in rng.integers(0, 1 << 31, 2000)]
    for n in ns:
        if 0 <= n < (1 << 31):
            assert fdiv(n, m, s) == n // d, (n, d)
