"""FastDiv (zillaphp_b200/csrc/common.cuh): division by a launch-time divisor
as a multiply and a shift (Granlund and Montgomery 1994, Theorem 4.2 with
N = 31), restated here with the same integer steps and checked against
floor division for every divisor 1..4096, the conv geometries' divisors and
extremes, on the edge numerators around multiples of d and up to 2^31 - 1."""
import numpy as np


def fastdiv(d):
    l = 0
    while (1 << l) < d:
        l += 1
    sh = 31 + l
    m = ((1 << sh) + d - 1) // d
    assert m < (1 << 32) and m >= (1 << 31)
    return m, sh


def check(d, ns):
    m, sh = fastdiv(d)
    ns = np.asarray(ns, dtype=object)
    got = [(int(n) * m) >> sh for n in ns]
    want = [int(n) // d for n in ns]
    assert got == want, d


def test_small_divisors_exhaustive_edges():
    top = (1 << 31) - 1
    for d in range(1, 4097):
        ks = [0, 1, 2, 3, 7, 1000, top // d - 1, top // d]
        ns = {0, top, d - 1, d}
        for k in ks:
            for off in (-1, 0, 1):
                n = k * d + off
                if 0 <= n <= top:
                    ns.add(n)
        check(d, sorted(ns))


def test_conv_geometry_divisors_random():
    rng = np.random.default_rng(0)
    top = (1 << 31) - 1
    divs = [784, 28, 196, 14, 49, 7, 6464, 101, 1600, 50, 400, 25, 96, 12, 9, 3, 6784, 26476544,
            (1 << 30) + 1, (1 << 31) - 1, 1 << 30, 65537]
    for d in divs:
        ns = list(rng.integers(0, top, 2000)) + [top, d * (top // d), d * (top // d) - 1]
        check(d, [n for n in ns if 0 <= n <= top])
