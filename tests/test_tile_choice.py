"""The tensor-core kernel's tile and split choice (host logic, no GPU), pinned on the BASELINE shapes.

Each expectation restates a rule of the router in the library's tile choice: swapped operands with
the narrowest tile covering M for M <= 64, split-K doubling while the grid stays within ~320 CTAs;
for larger M, 128-wide weight tiles widened to 192 / 256 only while the grid would exceed one wave of
148 CTAs, CTA-pair tiles for nibble weights past one wave, split-K for grids of at most 32 / 64
tiles; nibble weights at M <= 16 whose unsplit grid exceeds 296 tiles take the 2-stage ring with a
2-way split; long int8 rows (K >= 6144) at M <= 32 take a 6-deep ring.
"""
import ctypes

import pytest

import ork_b200

F16, I8, U4, NF4 = 0, 1, 2, 3


def choice(fmt, M, K, N):
    out = (ctypes.c_int * 5)()
    assert ork_b200.lib().ork_b200_tc_choice(fmt, M, K, N, out) == 0
    return list(out)


@pytest.fixture(autouse=True)
def no_tuning_variables(monkeypatch):
    for v in ("ORKB_TC_TN", "ORKB_TC_NA", "ORKB_TC_STAGES", "ORKB_TC_PAIR", "ORKB_TC_SK"):
        monkeypatch.delenv(v, raising=False)


@pytest.mark.parametrize("fmt,M,K,N,want", [
    # [swap, tile width, K split, ring depth (0 = default), CTA pair]
    (I8, 8, 6144, 2048, [1, 16, 8, 6, 0]),        # decode-sized int8, long rows: 6-deep ring
    (I8, 8, 2048, 6144, [1, 16, 4, 0, 0]),        # 48 tiles: split while <= 320 CTAs
    (I8, 128, 6144, 2048, [0, 128, 4, 0, 0]),     # 16 tiles, long K
    (I8, 512, 6144, 2048, [0, 128, 2, 0, 0]),     # 64 tiles, K of 48 blocks
    (I8, 512, 2048, 6144, [0, 192, 1, 0, 0]),     # 192 tiles of 128 > 148: widened to 192 (128 tiles)
    (I8, 512, 2048, 2048, [0, 128, 1, 0, 0]),     # 64 tiles, K of 16 blocks: too short to split
    (F16, 64, 2048, 6144, [1, 64, 4, 0, 0]),      # fp16 decode-sized batch
    (NF4, 8, 8192, 10240, [1, 16, 4, 0, 0]),      # 70B QKV at M = 8: 80 tiles x 4 = 320 CTAs
    (NF4, 8, 8192, 57344, [1, 16, 2, 2, 0]),      # 70B gate+up at M = 8: 448 tiles -> 2-stage ring, split 2
    (U4, 32, 8192, 57344, [1, 32, 1, 0, 0]),      # the wide-grid rule is for M <= 16 only
    (NF4, 256, 2048, 12288, [0, 192, 1, 0, 1]),   # nibble weights past one wave: CTA-pair 256 x 192
])
def test_tile_choice(fmt, M, K, N, want):
    assert choice(fmt, M, K, N) == want


@pytest.mark.parametrize("tiles,want", [(296, [1, 16, 1, 0, 0]), (297, [1, 16, 2, 2, 0])])
def test_wide_nibble_grid_boundary(tiles, want):
    for fmt in (U4, NF4):
        assert choice(fmt, 8, 1056, tiles * 128) == want


def test_tuning_variables_are_honoured(monkeypatch):
    monkeypatch.setenv("ORKB_TC_SK", "3")
    monkeypatch.setenv("ORKB_TC_STAGES", "2")
    assert choice(NF4, 8, 4128, 384)[2:4] == [3, 2]


def test_bad_arguments_refused():
    L = ork_b200.lib()
    out = (ctypes.c_int * 5)()
    assert L.ork_b200_tc_choice(4, 8, 2048, 2048, out) == -1
    assert L.ork_b200_tc_choice(I8, 0, 2048, 2048, out) == -1
    assert L.ork_b200_tc_choice(I8, 8, 2048, 2048, None) == -1
