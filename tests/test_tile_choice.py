"""The kernel choices of the router (host logic, no GPU), pinned on the BASELINE shapes.

Tensor-core tiles:
Each expectation restates a rule of the router in the library's tile choice: swapped operands with
the narrowest tile covering M for M <= 64, split-K doubling while the grid stays within ~320 CTAs;
for larger M, 128-wide weight tiles widened to 192 / 256 only while the grid would exceed one wave of
148 CTAs, CTA-pair tiles for nibble weights past one wave, then the largest split of {2, 3, 4, 6}
that keeps tiles x split <= 132 CTAs and at least 4 k-blocks per split (2 at most for CTA pairs); nibble weights at M <= 16 whose unsplit grid exceeds 296 tiles take the 2-stage ring with a
2-way split; long int8 rows (K >= 6144) at M <= 32 take a 6-deep ring; narrow nibble weights at
M <= 32 with K >= 6144 that reach 8 splits continue to 16 (or 12) splits through the tile flags while the
grid stays within 256 CTAs. int8 weights at larger M whose
grid can fit one wave take the width (64-256) and split (1-6, >= 5 k-blocks each, <= 148 CTAs) that
minimise the fitted cost 4.17 + 0.0088 * operand KB per CTA + 0.0052 * C KB per CTA + 0.166 * MB of C
written by all splits (microseconds).

Decode GEMV (M <= 8 per pass): the staged kernel (8 channels per CTA, whole rows in shared memory)
unless its rows and 8 activation rows exceed 196 KB, or M > 4 with K >= 8192, or nibble weights with
short rows (K <= 2048, N <= 8192); the direct kernel then takes 4 channels per warp (2 for NF4 at
M > 4, and for the short nibble rows).
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
    for v in ("ORKB_TC_TN", "ORKB_TC_NA", "ORKB_TC_STAGES", "ORKB_TC_PAIR", "ORKB_TC_SK", "ORKB_TC_FLAGS",
              "ORKB_GEMV_KIND", "ORKB_GEMV_CPW", "ORKB_GEMV_TR", "ORKB_GEMV_NW"):
        monkeypatch.delenv(v, raising=False)


@pytest.mark.parametrize("fmt,M,K,N,want", [
    # [swap, tile width, K split, ring depth (0 = default), CTA pair]
    (I8, 8, 6144, 2048, [1, 16, 8, 6, 0]),        # decode-sized int8, long rows: 6-deep ring
    (I8, 8, 2048, 6144, [1, 16, 4, 0, 0]),        # 48 tiles: split while <= 320 CTAs
    (I8, 128, 6144, 2048, [0, 64, 4, 0, 0]),      # cost model: 32 tiles of 64 x split 4 (128 CTAs)
    (I8, 128, 2048, 6144, [0, 128, 3, 0, 0]),     # 48 tiles x split 3 = 144 CTAs (no cluster cap)
    (I8, 128, 2048, 2048, [0, 64, 3, 0, 0]),      # 32 tiles of 64 x split 3 (5 k-blocks per split)
    (I8, 512, 6144, 2048, [0, 192, 3, 0, 0]),     # 44 tiles of 192 x split 3 = 132 CTAs
    (I8, 512, 2048, 6144, [0, 192, 1, 0, 0]),     # 128 tiles of 192, unsplit
    (I8, 512, 2048, 2048, [0, 128, 2, 0, 0]),     # 64 tiles: split 2 (128 CTAs)
    (F16, 64, 2048, 6144, [1, 64, 4, 0, 0]),      # fp16 decode-sized batch
    (NF4, 8, 8192, 10240, [1, 16, 4, 0, 0]),      # 70B QKV at M = 8: 80 tiles x 4 = 320 CTAs
    (NF4, 8, 8192, 57344, [1, 16, 2, 2, 0]),      # 70B gate+up at M = 8: 448 tiles -> 2-stage ring, split 2
    (NF4, 8, 8192, 1024, [1, 16, 16, 0, 0]),      # 8-GPU shard of O: split 16 through the tile flags
    (NF4, 8, 8192, 2560, [1, 16, 12, 0, 0]),      # 4-GPU shard of QKV: 20 tiles, split 12 (240 CTAs)
    (NF4, 8, 28672, 4096, [1, 16, 8, 0, 0]),      # 2-GPU shard of down: 32 tiles, 8 in clusters
    (U4, 32, 6144, 2048, [1, 32, 16, 0, 0]),      # configs[2] w4a8 M = 32: 16 tiles x 16 splits
    (I8, 32, 6144, 2048, [1, 32, 8, 6, 0]),       # int8 stays at 8 splits in clusters
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


def gemv_choice(fmt, M, K, N):
    out = (ctypes.c_int * 4)()
    assert ork_b200.lib().ork_b200_gemv_choice(fmt, M, K, N, out) == 0
    return list(out)


@pytest.mark.parametrize("fmt,M,K,N,want", [
    # [direct, channels per warp (direct), channels per CTA (staged), activation rows per pass]
    (NF4, 1, 28672, 8192, [1, 4, 0, 1]),    # 70B down projection: rows too long to stage with 8 A rows
    (NF4, 1, 28672, 4096, [1, 1, 0, 1]),    # ... its 2-GPU shard: direct, one channel per warp (512 CTAs)
    (NF4, 1, 28672, 2048, [0, 0, 8, 1]),    # ... its 4-GPU shard: staged with the one A row (N / 8 < 296)
    (NF4, 1, 28672, 1024, [0, 0, 8, 1]),    # ... and its 8-GPU shard
    (NF4, 8, 28672, 2048, [1, 4, 0, 8]),    # eight A rows do not fit beside the weight rows
    (NF4, 1, 8192, 57344, [0, 0, 8, 1]),    # 70B gate+up at M = 1: staged
    (NF4, 8, 8192, 10240, [1, 2, 0, 8]),    # M = 8, K >= 8192: direct, 2 NF4 channels per warp
    (I8, 8, 8192, 8192, [1, 4, 0, 8]),
    (I8, 1, 6144, 2048, [0, 0, 8, 1]),      # configs[1] decode shapes: staged
    (I8, 3, 2048, 2048, [0, 0, 8, 4]),
    (I8, 2, 2048, 6144, [0, 0, 8, 2]),
    (U4, 1, 2048, 6144, [1, 2, 0, 1]),      # short nibble rows
    (U4, 1, 2048, 12288, [0, 0, 8, 1]),     # ... unless N > 8192
    (F16, 1, 2048, 6144, [0, 0, 8, 1]),     # configs[0] M = 1
    (F16, 4, 16384, 2048, [1, 4, 0, 4]),    # fp16 rows of 32 KB: too long to stage
])
def test_gemv_choice(fmt, M, K, N, want):
    assert gemv_choice(fmt, M, K, N) == want


def test_gemv_choice_refuses_bad_arguments():
    L = ork_b200.lib()
    out = (ctypes.c_int * 4)()
    assert L.ork_b200_gemv_choice(I8, 9, 2048, 2048, out) == -1  # more than one decode pass
    assert L.ork_b200_gemv_choice(5, 1, 2048, 2048, out) == -1
    assert L.ork_b200_gemv_choice(I8, 1, 2048, 2048, None) == -1
