"""Pins of the oracle (the CPU restatement of the reference's query path).

The reference has no golden vectors for this path and cannot be built here, so each oracle
component is checked against an independent known answer: published splitmix64 outputs, the
closed form of the Sylvester-Hadamard matrix, the reference's own unit tests
(src/quantize.rs:445-492), hand-computed FastScan tables and block layouts, and agreement of its
scalar and AVX2 FastScan kernels (src/quantize.rs:335-386).
"""
from __future__ import annotations

from fractions import Fraction

import numpy as np
import pytest

import oracle


def test_splitmix64_published_values():
    # Vigna's splitmix64 reference outputs for seed 0 (and the commonly quoted seed-1234567 start)
    assert [int(x) for x in oracle.splitmix64(0, 3)] == [0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4, 0x06C45D188009454F]
    got = [int(x) for x in oracle.splitmix64(1234567, 5)]
    assert got == [6457827717110365317, 3203168211198807973, 9817491932198370423, 4593380528125082431,
                   16408922859458223821]


def test_make_signs_follow_low_bit_of_splitmix64():
    dp, seed = 128, 0x5EED
    s = oracle.make_signs(dp, seed)
    raw = oracle.splitmix64(seed, 2 * dp)
    assert np.array_equal(s, np.where((raw & np.uint64(1)) == 0, 1.0, -1.0).astype(np.float32))


@pytest.mark.parametrize("n", [64, 512, 1024])
def test_fht_of_unit_vectors_is_the_hadamard_row(n):
    s = np.float32(1.0) / np.sqrt(np.float32(n))
    for i in (0, 1, 5, n - 1):
        e = np.zeros(n, np.float32)
        e[i] = 1.0
        out = oracle.fht(e)
        j = np.arange(n)
        sign = np.array([(-1) ** bin(i & int(x)).count("1") for x in j], np.float32)
        assert np.array_equal(out, sign * s)


def test_fht_is_orthonormal():  # quantize.rs:449-457
    a = np.sin(np.arange(64, dtype=np.float32) * np.float32(0.37)).astype(np.float32)
    b = oracle.fht(a)
    assert abs(float((a * a).sum()) - float((b * b).sum())) < 1e-3


def test_rotation_preserves_inner_product():  # quantize.rs:459-472
    dim = 64
    signs = oracle.make_signs(dim, 42)
    a = np.cos(np.arange(dim, dtype=np.float32) * np.float32(0.11)).astype(np.float32)
    b = np.sin(np.arange(dim, dtype=np.float32) * np.float32(0.23)).astype(np.float32)
    ra, rb = oracle.rotate(a, signs, dim), oracle.rotate(b, signs, dim)
    assert abs(float(a @ b) - float(ra @ rb)) < 1e-3


def test_hamming_orders_like_cosine():  # quantize.rs:474-492
    dim = 256
    signs = oracle.make_signs(dim, 7)
    q = np.sin(np.arange(dim, dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    codes = oracle.encode(np.vstack([q, q + 0.01, -q]), signs, dim, dim // 64)

    def ham(a, b):
        return sum(bin(int(x) ^ int(y)).count("1") for x, y in zip(a, b))

    assert ham(codes[0], codes[1]) < ham(codes[0], codes[2])


def _f32_round(x: Fraction) -> np.float32:
    """Correctly rounded f32 of an exact rational (ties to even)."""
    f = np.float32(float(x))
    lo, hi = np.nextafter(f, np.float32(-np.inf)), np.nextafter(f, np.float32(np.inf))
    best = min((lo, f, hi), key=lambda c: (abs(Fraction(float(c)) - x), int(np.float32(c).view(np.uint32)) & 1))
    return np.float32(best)


def test_fsquery_lut_by_hand():
    # A rotated vector whose tables are easy to compute exactly (quantize.rs:279-313).
    nw = 1
    rot = np.zeros(64, np.float32)
    rot[:8] = [0.5, -0.25, 0.125, 1.0, 0.0, 0.0, -0.5, 0.75]
    lut, delta, bias = oracle.fsquery(rot, nw)
    raws, mins, rng_max = [], [], Fraction(0)
    for j in range(16):
        x = [Fraction(float(rot[4 * j + t])) for t in range(4)]
        raw = [sum((-x[t] if (e >> t) & 1 else x[t]) for t in range(4)) for e in range(16)]
        raws.append(raw)
        mins.append(min(raw))
        rng_max = max(rng_max, max(raw) - min(raw))
    d = _f32_round(Fraction(float(_f32_round(rng_max))) / 255)
    assert np.float32(delta) == d
    exp = np.zeros(256, np.uint8)
    for j in range(16):
        for e in range(16):
            v = (Fraction(float(_f32_round(raws[j][e] - mins[j]))) / Fraction(float(d)))
            q = int(Fraction(float(_f32_round(v))) + Fraction(1, 2))  # values are positive: half away = floor(x+.5)
            exp[16 * j + e] = min(max(q, 0), 255)
    assert np.array_equal(lut, exp)
    assert np.float32(bias) == np.float32(sum(float(m) for m in mins))


def test_fs_pack_block_layout_by_hand():
    # lane i's code has nibble j == (i + j) % 16 (quantize.rs:238-250 layout)
    nw = 1
    codes = np.zeros((20, nw), np.uint64)
    for i in range(20):
        v = 0
        for j in range(16):
            v |= ((i + j) % 16) << (4 * j)
        codes[i, 0] = v
    blk = oracle.fs_pack_block(codes, nw)
    for p in range(8):
        for half in range(2):
            j = 2 * p + half
            for i in range(16):
                lo = (i + j) % 16
                hi = ((i + 16) + j) % 16 if i + 16 < 20 else 0
                assert blk[p * 32 + half * 16 + i] == lo | (hi << 4)


@pytest.mark.parametrize("nw", [1, 4, 8, 12])
def test_block_sums_avx2_equals_scalar_equals_definition(nw):
    rng = np.random.default_rng(nw)
    codes = rng.integers(0, 2**63, size=(32, nw), dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, (32, nw),
                                                                                              dtype=np.uint64)
    lut = rng.integers(0, 256, nw * 16 * 16, dtype=np.uint8)
    blk = oracle.fs_pack_block(codes, nw)
    a = oracle.fs_block_sums(blk, lut, nw, avx2=True)
    s = oracle.fs_block_sums(blk, lut, nw, avx2=False)
    ref = np.zeros(32, np.int64)
    for i in range(32):
        for j in range(nw * 16):
            nibv = (int(codes[i, j >> 4]) >> (4 * (j & 15))) & 0xF
            ref[i] += int(lut[16 * j + nibv])
    assert np.array_equal(a, s) and np.array_equal(a.astype(np.int64), ref)


def test_hamming_cutoff_keeps_ties():  # index.rs:86-104
    hs = np.array([5, 3, 3, 9, 3, 1], np.uint16)
    assert oracle.hamming_cutoff(hs, 1, 64) == 1
    assert oracle.hamming_cutoff(hs, 2, 64) == 3  # ties at 3 are all within the cut
    assert oracle.hamming_cutoff(hs, 5, 64) == 5
    assert oracle.hamming_cutoff(hs, 7, 64) == 64
    assert oracle.hamming_cutoff(hs, 0, 64) == 0


def test_keep_smallest_encounter_order():  # tree.rs:120-159
    h = np.array([4, 2, 4, 1, 4, 7], np.uint32)
    ids = np.arange(6, dtype=np.uint32) + 100
    assert oracle.keep_smallest(h, ids, 3, 64).tolist() == [100, 101, 103]
    assert oracle.keep_smallest(h, ids, 4, 64).tolist() == [100, 101, 102, 103]
    assert oracle.keep_smallest(h, ids, 6, 64).tolist() == ids.tolist()


def _fma_f32(a, b, c):
    return _f32_round(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def test_dot_f32_lane_order():  # index.rs:136-152 with hsum_ps :58-65
    rng = np.random.default_rng(5)
    for n in (8, 24, 19):
        a = rng.standard_normal(n).astype(np.float32)
        b = rng.standard_normal(n).astype(np.float32)
        acc = [np.float32(0.0)] * 8
        full = n & ~7
        for i in range(0, full, 8):
            for lane in range(8):
                acc[lane] = _fma_f32(a[i + lane], b[i + lane], acc[lane])
        s0 = np.float32(acc[0] + acc[4])
        s1 = np.float32(acc[1] + acc[5])
        s2 = np.float32(acc[2] + acc[6])
        s3 = np.float32(acc[3] + acc[7])
        s = np.float32(np.float32(s0 + s2) + np.float32(s1 + s3))
        for i in range(full, n):
            s = np.float32(s + np.float32(a[i] * b[i]))
        assert oracle.dot_f32(a, b) == s
