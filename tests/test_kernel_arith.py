"""The integer arithmetic of the FastScan sums and of the distance select, restated on the CPU.

The device code (maivs_b200/csrc/cuda/kernels.cu) looks up 8 members' table bytes with byte
permutes (`lut16x8`), adds the looked-up bytes as whole 32-bit words and widens only the odd
bytes (`GroupAcc`), and selects the kth smallest distance with two histograms over the keys' own
range (`block_select_d`). These tests check each identity the kernels rely on against the
definition, on random inputs and on the edge values (all 255s, npos = 256, ties); the GPU tests
then check the kernels themselves against the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest

MASK32 = 0xFFFFFFFF


def prmt(a: int, b: int, sel: int) -> int:
    """prmt.b32 in its generic mode with bit 3 of every selector nibble clear."""
    src = [(a >> (8 * i)) & 0xFF for i in range(4)] + [(b >> (8 * i)) & 0xFF for i in range(4)]
    out = 0
    for i in range(4):
        nib = (sel >> (4 * i)) & 0xF
        assert nib & 8 == 0, "a selector with the sign-replicate bit set"
        out |= src[nib & 7] << (8 * i)
    return out


def lut16x8(t: list[int], w: int) -> tuple[int, int]:
    """The device's lookup of 8 nibbles of w in the 16-byte table t (four little-endian words)."""
    s3 = w & 0x77777777
    pk = ((w >> 1) & 0x44444444) | 0x32103210
    r0 = prmt(prmt(t[0], t[1], s3), prmt(t[2], t[3], s3), pk)
    s3h, pkh = s3 >> 16, pk >> 16
    r1 = prmt(prmt(t[0], t[1], s3h), prmt(t[2], t[3], s3h), pkh)
    return r0, r1


def table_words(tab: np.ndarray) -> list[int]:
    return [int.from_bytes(bytes(tab[4 * i:4 * i + 4].tolist()), "little") for i in range(4)]


def test_lut16x8_is_the_table_lookup():
    rng = np.random.default_rng(1)
    for _ in range(2000):
        tab = rng.integers(0, 256, 16, dtype=np.uint8)
        w = int(rng.integers(0, 2**32))
        r0, r1 = lut16x8(table_words(tab), w)
        got = [(r0 >> (8 * b)) & 0xFF for b in range(4)] + [(r1 >> (8 * b)) & 0xFF for b in range(4)]
        want = [int(tab[(w >> (4 * b)) & 0xF]) for b in range(8)]
        assert got == want


class GroupAcc:
    """all += looked-up word (mod 2^32); odd += bytes 1 and 3 widened; even = all - (odd << 8)."""

    def __init__(self):
        self.all0 = self.odd0 = self.all1 = self.odd1 = 0

    def add(self, r0: int, r1: int):
        self.all0 = (self.all0 + r0) & MASK32
        self.odd0 = (self.odd0 + prmt(r0, 0, 0x4341)) & MASK32
        self.all1 = (self.all1 + r1) & MASK32
        self.odd1 = (self.odd1 + prmt(r1, 0, 0x4341)) & MASK32

    def finish(self) -> list[int]:
        e0 = (self.all0 - (self.odd0 << 8)) & MASK32
        e1 = (self.all1 - (self.odd1 << 8)) & MASK32
        acc = [prmt(e0, self.odd0, 0x5410), prmt(e0, self.odd0, 0x7632),
               prmt(e1, self.odd1, 0x5410), prmt(e1, self.odd1, 0x7632)]
        return [(acc[b >> 1] >> (16 * (b & 1))) & 0xFFFF for b in range(8)]


@pytest.mark.parametrize("npos", [16, 96, 192, 256])
def test_group_sums_without_widening_every_byte(npos):
    rng = np.random.default_rng(npos)
    for trial in range(20):
        # trial 0: every looked-up byte 255, the largest sums (255 x 256 = 65,280 < 2^16)
        lut = np.full((npos, 16), 255, np.uint8) if trial == 0 else rng.integers(0, 256, (npos, 16), dtype=np.uint8)
        words = rng.integers(0, 2**32, npos, dtype=np.uint64)
        acc = GroupAcc()
        for j in range(npos):
            acc.add(*lut16x8(table_words(lut[j]), int(words[j])))
        want = [sum(int(lut[j, (int(words[j]) >> (4 * b)) & 0xF]) for j in range(npos)) for b in range(8)]
        assert acc.finish() == want


def select_d(d: np.ndarray, kth: int) -> int:
    """block_select_d: the kth smallest (1-based) of distances below 2^16 by two histograms of at
    most 256 bins over [lo, hi]."""
    lo, hi = int(d.min()), int(d.max())
    sh = 0
    while ((hi - lo) >> sh) > 255:
        sh += 1
    rel = d.astype(np.int64) - lo
    hist = np.bincount(rel >> sh, minlength=256)
    assert hist.size <= 256
    cum = np.cumsum(hist)
    b = int(np.searchsorted(cum, kth))  # first bin whose running count reaches kth
    rem = kth - (int(cum[b - 1]) if b else 0)
    if sh == 0:
        return lo + b
    inbin = rel[(rel >> sh) == b] & ((1 << sh) - 1)
    hist2 = np.bincount(inbin, minlength=1 << sh)
    assert hist2.size <= 256
    sub = int(np.searchsorted(np.cumsum(hist2), rem))
    return lo + (b << sh) + sub


def test_select_d_is_the_kth_smallest():
    rng = np.random.default_rng(7)
    for t in range(500):
        n = int(rng.integers(1, 3000))
        spread = int(rng.choice([1, 5, 300, 5000, 65535]))
        base = int(rng.integers(0, 65536 - spread))
        d = base + rng.integers(0, spread, n)
        if t % 5 == 0:  # heavy ties at one value
            d[: n // 2] = d[0]
        kth = int(rng.integers(1, n + 1))
        assert select_d(d, kth) == int(np.sort(d)[kth - 1])
