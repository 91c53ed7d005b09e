"""Persisted tiled weights and grouped scales on the B200, through the C ABI.

Persistence (ork-driver include/ork/weights.h:159-269): ork_w_dump of every weight kind equals the
host-side ork_*_w_dump_cpu bytes for the same B, reloads through ork_*_mm_load to a weight whose results
equal the original's and the oracle's, and every header refusal the reference defines turns a load into
NULL. Grouped scales (src/npu/core/buf.c:501-520): ork_i4_mm_run_grouped and ork_i8_mm_run_grouped equal
the restated fp32 accumulate bit for bit, and the fp32 results recorded from the reference itself.
"""
import ctypes as C
import hashlib
import json
import os

import numpy as np
import pytest

import oracle_ffi as of
import ork_b200
from make_fixtures import grouped_inputs

pytestmark = pytest.mark.gpu
HDR = 4096
_p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731


def _bits_equal(a, b):
    return np.array_equal(np.ascontiguousarray(a, np.float32).view(np.uint32),
                          np.ascontiguousarray(b, np.float32).view(np.uint32))


def test_i8_dump_equals_cpu_dump_and_reloads(ctx):
    K, N = 1024, 384
    rng = np.random.default_rng(1)
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    w = ctx.i8_pack(B)
    blob = w.pack_dump()
    assert blob is not None and blob.size == HDR + K * N
    assert np.array_equal(blob, ctx.dump_cpu(B, "i8"))
    w2 = ctx.load(blob, K, N, "i8")
    assert w2
    try:
        for M in (1, 7, 130):
            A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
            rc, Cm = ctx.run(w2, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, B)), M
        assert np.array_equal(w2.pack_dump(), blob)  # re-dumps byte-identically
    finally:
        w.free()
        w2.free()


def test_i4_dump_equals_cpu_dump_and_reloads(ctx):
    K, N = 2048, 256
    rng = np.random.default_rng(2)
    B = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    w = ctx.i4_pack(B)
    blob = w.pack_dump()
    assert blob.size == HDR + K * N // 2 and np.array_equal(blob, ctx.dump_cpu(B, "i4"))
    w2 = ctx.load(blob, K, N, "i4")
    assert w2
    try:
        for M in (1, 40):
            A = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
            rc, Cm = ctx.run(w2, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, B)), M
    finally:
        w.free()
        w2.free()


def test_f16_dump_reloads(ctx):
    K, N = 512, 48
    rng = np.random.default_rng(3)
    B = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    w = ctx.f16_pack(B)
    blob = w.pack_dump()
    assert blob.size == HDR + 2 * K * N
    assert np.array_equal(blob[HDR:].view(np.float16).reshape(N, K), B.T)
    w2 = ctx.load(blob, K, N, "f16")
    assert w2
    try:
        A = rng.uniform(-1, 1, size=(5, K)).astype(np.float16)
        rc1, C1 = ctx.run(w, A)
        rc2, C2 = ctx.run(w2, A)
        assert rc1 == 0 and rc2 == 0 and _bits_equal(C1, C2)
    finally:
        w.free()
        w2.free()


@pytest.mark.parametrize("nf4", [False, True])
def test_int4_store_dumps_as_int8_codes(ctx, env_clean, nf4):
    """An ork_i4a8 weight persists as its int8 codes (what the NPU's resident tiles hold) and reloads
    through ork_i8_mm_load as a plain int8 weight with identical results."""
    if nf4:
        env_clean.setenv("ORK_NF4", "1")
    K, N = 1024, 256
    rng = np.random.default_rng(4)
    f32 = rng.standard_normal((N, K), dtype=np.float32)
    w, _ = ctx.i4a8_pack(f32)
    codes, _, _ = of.i4a8_blob_codes(w.dump(), K, N)
    blob = w.pack_dump()
    assert blob.size == HDR + K * N
    assert np.array_equal(blob[HDR:].view(np.int8).reshape(N, K), codes.T)
    w2 = ctx.load(blob, K, N, "i8")
    assert w2
    try:
        A = rng.integers(-128, 128, size=(33, K), dtype=np.int8)
        rc1, C1 = ctx.run(w, A)
        rc2, C2 = ctx.run(w2, A)
        assert rc1 == 0 and rc2 == 0 and np.array_equal(C1, C2) and np.array_equal(C1, of.gemm_i32(A, codes))
    finally:
        w.free()
        w2.free()


def test_loads_refuse_foreign_or_mismatched_blobs(ctx):
    K, N = 256, 128
    B = np.random.default_rng(5).integers(-8, 8, size=(K, N), dtype=np.int8)
    b8, b4 = ctx.dump_cpu(B, "i8"), ctx.dump_cpu(B, "i4")
    L = ctx.L

    def load(fn, blob, k=K, n=N, size=None):
        return fn(ctx.ctx, k, n, _p(blob), blob.nbytes if size is None else size)

    assert not load(L.ork_i4_mm_load, b8)           # dtype int8 blob into the int4 loader (SHAPE)
    assert not load(L.ork_i8_mm_load, b4)
    assert not load(L.ork_f16_mm_load, b8)
    assert not load(L.ork_i8_mm_load, b8, k=K + 32)  # shape
    assert not load(L.ork_i8_mm_load, b8, size=b8.nbytes - 1)  # truncated payload
    assert not load(L.ork_i8_mm_load, b8, size=HDR - 1)        # SHORT
    for off, bit in ((0, 1), (4, 2), (8, 1), (24, 1)):          # UNSTAMPED, FORMAT, CAPS, header size
        bad = b8.copy()
        bad[off] ^= bit
        assert not load(L.ork_i8_mm_load, bad), off
    w = load(L.ork_i8_mm_load, b8)
    assert w
    L.ork_mm_free(ctx.ctx, w)
    # the tiled loader takes W4A4 blobs only
    assert not L.ork_i4a8_mm_load_tiled(ctx.ctx, K, N, _p(b8), b8.nbytes, 32)


@pytest.mark.parametrize("K,G", [(2048, 32), (2048, 128), (2048, 1024), (2016, 96), (3072, 384)])
def test_i4_grouped_exact(ctx, K, G):
    """Group sizes whose nibble bytes are one lane chunk (32), half a segment (128), several segments
    (1024), straddle lane sets (96 -> 48 bytes) or segments (384 -> 192 bytes)."""
    N = 320
    rng = np.random.default_rng(G)
    B = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    w = ctx.i4_pack_grouped(B, G)
    assert w
    try:
        for M in (1, 2, 5, 8, 13, 64):
            A = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
            aS = rng.uniform(1e-3, 3e-2, size=(M, K // G)).astype(np.float32)
            bS = rng.uniform(-3e-2, 3e-2, size=(K // G, N)).astype(np.float32)
            rc, Cm = ctx.run_grouped(w, A, aS, bS)
            assert rc == 0 and _bits_equal(Cm, of.gemm_grouped(A, B, G, aS, bS)), M
        # the grouped weight is still an ordinary W4A4 weight
        A = rng.integers(-8, 8, size=(3, K), dtype=np.int8)
        rc, Ci = ctx.run(w, A)
        assert rc == 0 and np.array_equal(Ci, of.gemm_i32(A, B))
    finally:
        w.free()


@pytest.mark.parametrize("G", [64, 256])
def test_i8_grouped_on_tiled_load_exact(ctx, G):
    """ork_i4_w_dump_cpu -> ork_i4a8_mm_load_tiled(G) -> ork_i8_mm_run_grouped with int8 activations."""
    K, N = 4096, 192
    rng = np.random.default_rng(G + 1)
    B = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    w = ctx.i4a8_load_tiled(ctx.dump_cpu(B, "i4"), K, N, G)
    assert w
    try:
        for M in (1, 4, 9):
            A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
            aS = rng.uniform(1e-3, 3e-2, size=(M, K // G)).astype(np.float32)
            bS = rng.uniform(1e-3, 3e-2, size=(K // G, N)).astype(np.float32)
            rc, Cm = ctx.run_grouped(w, A, aS, bS)
            assert rc == 0 and _bits_equal(Cm, of.gemm_grouped(A, B, G, aS, bS)), M
        A = rng.integers(-128, 128, size=(2, K), dtype=np.int8)
        rc, Ci = ctx.run(w, A)  # and an ordinary int8-compute weight
        assert rc == 0 and np.array_equal(Ci, of.gemm_i32(A, B))
    finally:
        w.free()


@pytest.mark.parametrize("kind", ["i8", "i8_g48", "nf4"])
def test_set_group_on_int8_compute_weights(ctx, env_clean, kind):
    K, N = (1056, 128) if kind == "i8_g48" else (1024, 128)
    rng = np.random.default_rng(7)
    if kind.startswith("i8"):
        B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
        w = ctx.i8_pack(B)
        codes_kn, G = B, (48 if kind == "i8_g48" else 16)
    else:
        env_clean.setenv("ORK_NF4", "1")
        w, _ = ctx.i4a8_pack(rng.standard_normal((N, K), dtype=np.float32))
        codes_kn, _, _ = of.i4a8_blob_codes(w.dump(), K, N)
        G = 128
    try:
        A = rng.integers(-128, 128, size=(3, K), dtype=np.int8)
        aS = np.ones((3, K // G), np.float32)
        bS = np.ones((K // G, N), np.float32)
        rc, _ = ctx.run_grouped(w, A, aS, bS)
        assert rc == -1  # no group size yet
        assert w.set_group(G) == 0
        aS = rng.uniform(1e-3, 3e-2, size=(3, K // G)).astype(np.float32)
        bS = rng.uniform(1e-3, 3e-2, size=(K // G, N)).astype(np.float32)
        rc, Cm = ctx.run_grouped(w, A, aS, bS)
        assert rc == 0 and _bits_equal(Cm, of.gemm_grouped(A, codes_kn, G, aS, bS))
        assert w.set_group(K - 32) == -1  # must divide K
        assert w.set_group(0) == 0
        rc, _ = ctx.run_grouped(w, A, aS, bS)
        assert rc == -1
    finally:
        w.free()


def test_grouped_refusals(ctx):
    L = ctx.L
    K, N = 256, 64
    B = np.zeros((K, N), np.int8)
    assert not L.ork_i4_mm_pack_grouped(ctx.ctx, K, N, _p(B), 48)   # G % 32
    assert not L.ork_i4_mm_pack_grouped(ctx.ctx, K, N, _p(B), 96)   # K % G
    assert not L.ork_i4_mm_pack_grouped(ctx.ctx, K, 96, _p(B), 32)  # N % 64
    wf = ctx.f16_pack(np.zeros((K, N), np.float16))
    assert wf.set_group(32) == -1
    wf.free()
    w = ctx.i4_pack_grouped(B, 32)
    A = np.zeros((2, K), np.int8)
    aS = np.ones((2, K // 32), np.float32)
    bS = np.ones((K // 32, N), np.float32)
    Cm = np.zeros((2, N), np.float32)
    assert L.ork_i8_mm_run_grouped(ctx.ctx, w.h, 2, _p(A), _p(aS), _p(bS), _p(Cm)) == -1  # dtype
    assert L.ork_i4_mm_run_grouped(ctx.ctx, w.h, 0, _p(A), _p(aS), _p(bS), _p(Cm)) == -1  # M
    shared = np.zeros(4096, np.int8)
    assert L.ork_i4_mm_run_grouped(ctx.ctx, w.h, 2, _p(shared), _p(aS), _p(bS),
                                   C.c_void_p(shared.ctypes.data + 64)) == -1  # A/C overlap
    assert L.ork_i4_mm_run_grouped(ctx.ctx, w.h, 2, _p(A), _p(aS), _p(bS), _p(Cm)) == 0
    w.free()


def test_grouped_reference_fixtures(ctx):
    fx = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_fixtures.json")))["grouped"]
    for name, c in fx.items():
        A, B, aS, bS = grouped_inputs(c["seed"], c["M"], c["K"], c["N"], c["G"], c["a_range"])
        if c["a_range"] == 8:
            w = ctx.i4_pack_grouped(B, c["G"])
        else:
            w = ctx.i4a8_load_tiled(ctx.dump_cpu(B, "i4"), c["K"], c["N"], c["G"])
        rc, Cm = ctx.run_grouped(w, A, aS, bS)
        w.free()
        assert rc == 0 and hashlib.sha256(Cm.tobytes()).hexdigest() == c["c_sha256"], name


def test_grouped_async_device_pointers(ctx):
    import torch

    L = ork_b200.lib()
    K, N, G, M = 2048, 256, 128, 4
    rng = np.random.default_rng(9)
    B = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    A = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
    aS = rng.uniform(1e-3, 3e-2, size=(M, K // G)).astype(np.float32)
    bS = rng.uniform(1e-3, 3e-2, size=(K // G, N)).astype(np.float32)
    w = ctx.i4_pack_grouped(B, G)
    dev = torch.device("cuda", L.ork_b200_device(ctx.ctx))
    tA, taS, tbS = (torch.from_numpy(x).to(dev) for x in (A, aS, bS))
    tC = torch.zeros((M, N), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    assert L.ork_b200_i4_mm_run_grouped_async(ctx.ctx, w.h, M, tA.data_ptr(), taS.data_ptr(), tbS.data_ptr(),
                                         tC.data_ptr()) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    assert _bits_equal(tC.cpu().numpy(), of.gemm_grouped(A, B, G, aS, bS))
    w.free()
