"""The integer arithmetic of the FastScan sums and of the distance select, restated on the CPU.

The device code (maivs_b200/csrc/cuda/dev_common.cuh, k_cellmajor.cu) looks up 8 members' table
bytes with byte permutes (`lut16x8`), adds the looked-up bytes as whole 32-bit words and widens
only the odd bytes (`GroupAcc`), and selects the kth smallest distance with two histograms over
the keys' own range (`block_select_d`). These tests check each identity the kernels rely on
against the definition, on random inputs and on the edge values (all 255s, npos = 256, ties), and
the index arithmetic of the rerank's work split, the tensor-core scan's epilogue and the rerank's
shared-memory fit; the GPU tests then check the kernels themselves against the oracle.
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


def test_rerank_stream_covers_every_candidate_once():
    """k_rerank_stream's work split: items of 16 candidate rows numbered by an exclusive prefix
    over the queries, stages of two items dealt to the CTAs in equal runs, thread t of a stage
    copying row 4 (t >> 5) + (t & 31) (lanes 0-3) and summing row t >> 3, both in item t >> 7.
    Every (query, candidate) pair is copied and summed exactly once, whatever the counts."""
    rng = np.random.default_rng(11)
    for trial in range(200):
        nq = int(rng.integers(1, 60))
        cand_n = rng.integers(0, 70, nq)
        if trial % 4 == 0:
            cand_n[rng.random(nq) < 0.5] = 0  # queries without candidates
        grid = int(rng.integers(1, 40))
        item_off = np.concatenate([[0], np.cumsum((cand_n + 15) // 16)])
        items = int(item_off[-1])
        nst = (items + 1) // 2
        copied, summed = {}, {}
        for b in range(grid):
            s0, s1 = nst * b // grid, nst * (b + 1) // grid
            for st in range(s0, s1):
                for t in range(256):
                    half = t >> 7
                    it = 2 * st + half
                    if it >= items:
                        continue
                    q = int(np.searchsorted(item_off, it, side="right") - 1)  # last q with item_off[q] <= it
                    lane, warp = t & 31, t >> 5
                    if lane < 4:
                        crow = warp * 4 + lane
                        assert crow >> 4 == half
                        r = (it - int(item_off[q])) * 16 + (crow & 15)
                        if r < cand_n[q]:
                            copied[(q, r)] = copied.get((q, r), 0) + 1
                    row = t >> 3
                    assert row >> 4 == half
                    if t & 7 == 0:  # the lane that stores the row's score
                        r = (it - int(item_off[q])) * 16 + (row & 15)
                        if r < cand_n[q]:
                            summed[(q, r)] = summed.get((q, r), 0) + 1
        want = {(q, r) for q in range(nq) for r in range(int(cand_n[q]))}
        assert set(copied) == want and set(copied.values()) <= {1}
        assert set(summed) == want and set(summed.values()) <= {1}


def test_shuffle_tree_is_the_reference_hsum_order():
    """k_rerank_stream closes a row's eight FMA chains (one per thread c of 8) with xor-shuffles
    over 4, 2, 1; lane 0 ends with ((c0 + c4) + (c2 + c6)) + ((c1 + c5) + (c3 + c7)), the
    reference's horizontal sum (index.rs:58-65), in f32 with the same roundings."""
    rng = np.random.default_rng(5)
    f32 = np.float32
    for _ in range(2000):
        c = (rng.standard_normal(8) * 10.0 ** rng.integers(-6, 6, 8)).astype(f32)
        v = c.copy()
        for off in (4, 2, 1):
            v = np.array([f32(v[i]) + f32(v[i ^ off]) for i in range(8)], dtype=f32)
        want = f32(f32(f32(c[0] + c[4]) + f32(c[2] + c[6])) + f32(f32(c[1] + c[5]) + f32(c[3] + c[7])))
        assert v[0].tobytes() == want.tobytes()


@pytest.mark.parametrize("ngroups", [1, 2, 4])
def test_scan_mma_epilogue_columns_cover_the_tile_once(ngroups):
    """k_scan_mma's epilogue: the tile's N = members rounded up to 16 columns are split over the
    column groups (warp / 4) in slices of cw = 16 * ceil(N / (16 * groups)) columns, loaded 16 at a
    time while the load starts below N. Every column below N is read by exactly one group, no load
    reaches past N (so never past the 256 allocated TMEM columns), and N is a legal kind::i8 width
    for M = 128 (a multiple of 16 from 16 to 256)."""
    for members in range(1, 600):
        for mt in range(0, members, 256):
            n_tile = (min(256, members - mt) + 15) & ~15
            assert n_tile % 16 == 0 and 16 <= n_tile <= 256
            cw = ((n_tile + 16 * ngroups - 1) // (16 * ngroups)) * 16
            seen = np.zeros(n_tile, dtype=int)
            for cq in range(ngroups):
                c0 = cw * cq
                cb = 0
                while cb < cw and c0 + cb < n_tile:
                    assert c0 + cb + 16 <= n_tile
                    seen[c0 + cb:c0 + cb + 16] += 1
                    cb += 16
            assert (seen == 1).all(), (members, mt, ngroups)


def test_rerank_stream_two_ctas_fit_one_sm():
    """The streamed rerank at d = 384 runs two CTAs of two 32-row stages per SM; its item table
    goes into shared memory only when both CTAs (stages, table, 1 KB reserved, 1.25 KB static) still
    fit the SM's 228 KB, otherwise into global memory (k_rerank_items)."""
    rstride = 384 + ((8 - 384 % 32) + 32) % 32
    stage = 32 * rstride * 4
    sm = 228 * 1024
    for nq in (1, 448, 552, 1000, 3000, 3455, 3456, 5000, 10000):
        items = (nq + 1) * 4
        local = 2 * (2 * stage + items + 2560) <= sm
        need = 2 * (2 * stage + (items if local else 0) + 1024 + 1280)
        assert need <= sm, nq  # two CTAs are resident whichever way the table goes
        assert local == (nq <= 3455), nq
