"""CUDA path vs the oracle, through the C ABI (needs a B200).

Integer paths (w8a8, w4a8 uniform / NF4, W4A4) must be bit-exact int32; fp16 must stay within
max|err| <= 1e-3 * sqrt(K) * max|A| * max|B| of the sequential-f32 reference (the tolerance of the
north star), and exact on integer-valued inputs. Also the reference's own goldens (examples/quant.c,
examples/test_matmul.c), the O4N1 round trip of examples/test_matmul.c:507-557, the overlap guard of
:559-589, the dtype / dimension refusals, and device-pointer (sync and async) runs.
"""
import numpy as np
import pytest

import oracle_ffi as of
import ork_b200
import reference_goldens as rg
from make_fixtures import seeded_imatrix, seeded_weights

pytestmark = pytest.mark.gpu

SHAPES = [(32, 64), (64, 128), (288, 192), (2048, 2048), (6144, 2048), (2048, 6144)]
MS = [1, 2, 3, 5, 8, 9, 17, 64]


def f16_tol(A, B):
    K = A.shape[1]
    return 1e-3 * np.sqrt(K) * float(np.abs(A.astype(np.float32)).max()) * float(np.abs(B.astype(np.float32)).max())


def rand_i8(rng, shape, lo=-128, hi=128):
    return rng.integers(lo, hi, size=shape, dtype=np.int8)


@pytest.mark.parametrize("K,N", SHAPES)
def test_i8_pack_run_exact(ctx, K, N):
    rng = np.random.default_rng(K * 7 + N)
    B = rand_i8(rng, (K, N))
    w = ctx.i8_pack(B)
    assert w
    res = w.resident().view(np.int8).reshape(N, K)
    assert np.array_equal(res, B.T)
    for M in MS:
        A = rand_i8(rng, (M, K))
        rc, Cm = ctx.run(w, A)
        assert rc == 0
        assert np.array_equal(Cm, of.gemm_i32(A, B)), M
    w.free()


@pytest.mark.parametrize("K,N", [(64, 32), (2048, 2048), (6144, 2048), (2048, 6144)])
def test_i8_pack_f32_codes_and_run_exact(ctx, K, N):
    f32 = seeded_weights(K + N, N, K)
    w, bs = ctx.i8_pack_f32(f32)
    codes, obs = of.i8_quant_f32(f32)
    assert np.array_equal(bs, obs)
    assert w.bscale() is None  # the scale goes only to bscale_out (src/npu/i8/pack.c:475-494)
    assert np.array_equal(w.resident().view(np.int8).reshape(N, K), codes)
    rng = np.random.default_rng(1)
    for M in (1, 8, 13):
        A = rand_i8(rng, (M, K), -127, 128)
        rc, Cm = ctx.run(w, A)
        assert rc == 0 and np.array_equal(Cm, of.gemm_i32_nk(A, codes))
    w.free()


@pytest.mark.parametrize("nf4", [False, True])
@pytest.mark.parametrize("use_im", [False, True])
@pytest.mark.parametrize("K,N", [(64, 32), (2048, 512), (6144, 2048), (2048, 12288)])
def test_i4a8_pack_run_exact(ctx, env_clean, nf4, use_im, K, N):
    if nf4:
        env_clean.setenv("ORK_NF4", "1")
    f32 = seeded_weights(3 * K + N, N, K)
    im = seeded_imatrix(K, K) if use_im else None
    w, bs = ctx.i4a8_pack(f32, im)
    assert w and w.quant_kind() == (1 if nf4 else 0)
    blob = of.i4a8_blob(f32, im, nf4=nf4)
    codes, obs, _ = of.i4a8_blob_codes(blob, K, N)
    assert np.array_equal(bs, obs) and np.array_equal(w.bscale(), obs)
    assert np.array_equal(w.resident(), blob[20 + 4 * N:])  # resident nibbles == O4N1 payload
    rng = np.random.default_rng(2)
    for M in (1, 3, 8, 32, 100, 256):
        A = rand_i8(rng, (M, K))
        rc, Cm = ctx.run(w, A)
        assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, codes)), M
    w.free()


@pytest.mark.parametrize("K,N", [(32, 64), (288, 128), (6144, 2048), (2048, 12288)])
def test_w4a4_exact(ctx, K, N):
    rng = np.random.default_rng(K + 3 * N)
    B = rand_i8(rng, (K, N), -8, 8)
    w = ctx.i4_pack(B)
    assert w
    for M in (1, 2, 7, 8, 32, 256):
        A = rand_i8(rng, (M, K), -8, 8)
        rc, Cm = ctx.run(w, A)
        assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, B)), M
    # full int8 range activations still accumulate exactly in int32 (no int16 saturation)
    A = rand_i8(rng, (3, K))
    rc, Cm = ctx.run(w, A)
    assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, B))
    w.free()


def test_w4a4_saturation_case(ctx):
    """examples/i4.c:37-58: the all -8 x -8 product that overflows int16 on the NPU stays exact here."""
    K, N = 1024, 64
    B = np.full((K, N), -8, np.int8)
    A = np.full((2, K), -8, np.int8)
    w = ctx.i4_pack(B)
    rc, Cm = ctx.run(w, A)
    assert rc == 0 and np.all(Cm == 64 * K)
    w.free()


@pytest.mark.parametrize("K,N", [(32, 16), (64, 48), (2048, 6144)])
def test_f16_within_tolerance(ctx, K, N):
    rng = np.random.default_rng(K + N)
    B = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    w = ctx.f16_pack(B)
    assert w
    for M in (1, 4, 8, 64):
        A = rng.uniform(-1, 1, size=(M, K)).astype(np.float16)
        rc, Cm = ctx.run(w, A)
        ref = of.gemm_f16(A, B)
        assert rc == 0
        assert np.abs(Cm - ref).max() <= f16_tol(A, B), M
    w.free()


def _run_golden(ctx, kind, Ms, K, N, A, B):
    w = ctx.f16_pack(B) if kind == "f16" else ctx.i8_pack(B)
    h = of.FNV_OFFSET
    for m in Ms:
        rc, Cm = ctx.run(w, A[:m], m)
        assert rc == 0
        h = of.fnv64(Cm, h)
    w.free()
    return h


@pytest.mark.parametrize("which", ["quant", "f16", "chain", "check_i8"])
def test_reference_goldens_on_gpu(ctx, which):
    for name, kind, Ms, K, N, A, B, gold in rg.cases(of.Lcg, which=(which,)):
        assert _run_golden(ctx, kind, Ms, K, N, A, B) == gold, name


@pytest.mark.parametrize("nf4", [True, False])
def test_o4n1_dump_load_roundtrip(ctx, env_clean, nf4):
    """examples/test_matmul.c:507-557 on the GPU path."""
    if nf4:
        env_clean.setenv("ORK_NF4", "1")
    K, N, M = 2048, 512, 8
    rng = np.random.default_rng(4)
    f32 = rng.standard_normal((N, K), dtype=np.float32)
    w, bs = ctx.i4a8_pack(f32)
    A = rand_i8(rng, (M, K), -127, 128)
    rc1, C_res = ctx.run(w, A)
    blob = w.dump()
    assert blob is not None and blob.size == 5 * 4 + N * 4 + K * N // 2
    assert np.array_equal(blob, of.i4a8_blob(f32, None, nf4=nf4))
    wl = ctx.i4a8_load(blob, K, N)
    assert wl
    rc2, C_str = ctx.run(wl, A)
    assert rc1 == 0 and rc2 == 0 and np.array_equal(C_res, C_str)
    assert np.array_equal(wl.dump(), blob)
    assert np.array_equal(wl.bscale(), bs)
    assert wl.quant_kind() == (1 if nf4 else 0)
    # a short cap returns 0, the size query the full size
    L = ork_b200.lib()
    assert L.ork_i4a8_w_dump(wl.h, blob.ctypes.data, blob.size - 1) == 0
    w.free()
    wl.free()


def test_null_imatrix_identity(ctx, env_clean):
    """examples/test_matmul.c:467-471: pack_im(NULL) scale is exactly absmax/7."""
    K, N = 2048, 64
    f32 = seeded_weights(6, N, K)
    w, bs = ctx.i4a8_pack(f32, None)
    mx = np.maximum(np.abs(f32).max(axis=1), np.float32(1e-9)).astype(np.float32)
    assert np.array_equal(bs, (mx / np.float32(7)).astype(np.float32))
    w.free()


def test_load_refuses_malformed_blobs(ctx):
    K, N = 64, 32
    blob = ork_b200.cpu_blob(seeded_weights(2, N, K))
    assert ctx.i4a8_load(blob, K, N)
    assert not ctx.i4a8_load(blob[:-1], K, N)
    assert not ctx.i4a8_load(np.concatenate([blob, blob[:1]]), K, N)
    assert not ctx.i4a8_load(blob, K, N + 32)
    for off, val in ((0, 0x4F344E32), (4, 2), (8, 96), (12, 64), (16, 7)):
        bad = blob.copy()
        bad[off:off + 4] = np.frombuffer(np.uint32(val).tobytes(), np.uint8)
        assert not ctx.i4a8_load(bad, K, N), off


def test_bad_dims_refused(ctx):
    L = ork_b200.lib()
    B = np.zeros(64 * 128, np.int8)
    f = np.zeros(64 * 128, np.float32)
    for K, N in ((33, 32), (32, 33), (16, 32)):
        assert not L.ork_i8_mm_pack(ctx.ctx, K, N, B.ctypes.data)
        assert not L.ork_i8_mm_pack_f32(ctx.ctx, K, N, f.ctypes.data, None)
        assert not L.ork_i4a8_mm_pack(ctx.ctx, K, N, f.ctypes.data, None)
    assert not L.ork_i4_mm_pack(ctx.ctx, 32, 32, B.ctypes.data)  # W4A4 needs N%64
    assert not L.ork_f16_mm_pack(ctx.ctx, 32, 24, B.ctypes.data)  # fp16 needs N%16


def test_dtype_mismatch_refused(ctx):
    rng = np.random.default_rng(0)
    wi8 = ctx.i8_pack(rand_i8(rng, (64, 64)))
    wi4 = ctx.i4_pack(rand_i8(rng, (64, 64), -8, 8))
    wf = ctx.f16_pack(np.zeros((64, 64), np.float16))
    L = ork_b200.lib()
    A = np.zeros((1, 64), np.int8)
    Ah = np.zeros((1, 64), np.float16)
    Cm = np.zeros((1, 64), np.int32)
    Cf = np.zeros((1, 64), np.float32)
    assert L.ork_i4_mm_run(ctx.ctx, wi8.h, 1, A.ctypes.data, Cm.ctypes.data) == -1
    assert L.ork_i8_mm_run(ctx.ctx, wi4.h, 1, A.ctypes.data, Cm.ctypes.data) == -1
    assert L.ork_f16_mm_run(ctx.ctx, wi8.h, 1, Ah.ctypes.data, Cf.ctypes.data) == -1
    assert L.ork_i8_mm_run(ctx.ctx, wf.h, 1, A.ctypes.data, Cm.ctypes.data) == -1
    assert L.ork_i8_mm_run(ctx.ctx, wi8.h, 0, A.ctypes.data, Cm.ctypes.data) == -1
    for w in (wi8, wi4, wf):
        w.free()


def test_overlap_guard(ctx):
    """examples/test_matmul.c:559-589: A and C sharing memory is refused with -1."""
    w = ctx.i8_pack(np.ones((32, 32), np.int8))
    shared = np.zeros(256, np.int8)
    L = ork_b200.lib()
    assert L.ork_i8_mm_run(ctx.ctx, w.h, 1, shared.ctypes.data, shared.ctypes.data + 16) == -1
    w.free()


def test_device_pointer_runs(ctx):
    import torch

    rng = np.random.default_rng(9)
    K, N, M = 2048, 2048, 8
    B = rand_i8(rng, (K, N))
    w = ctx.i8_pack(B)
    A = rand_i8(rng, (M, K))
    ref = of.gemm_i32(A, B)
    dA = torch.from_numpy(A).cuda()
    dC = torch.zeros((M, N), dtype=torch.int32, device="cuda")
    L = ork_b200.lib()
    torch.cuda.synchronize()
    assert L.ork_i8_mm_run(ctx.ctx, w.h, M, dA.data_ptr(), dC.data_ptr()) == 0
    assert np.array_equal(dC.cpu().numpy(), ref)
    dC.zero_()
    torch.cuda.synchronize()
    assert L.ork_b200_i8_mm_run_async(ctx.ctx, w.h, M, dA.data_ptr(), dC.data_ptr()) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    assert np.array_equal(dC.cpu().numpy(), ref)
    # async refuses host pointers' misalignment and overlap like the sync path
    assert L.ork_b200_i8_mm_run_async(ctx.ctx, w.h, M, dA.data_ptr() + 1, dC.data_ptr()) == -1
    w.free()


def test_kernels_are_launched(ctx):
    before = ctx.launches()
    w = ctx.i8_pack(np.ones((64, 64), np.int8))
    rc, Cm = ctx.run(w, np.ones((3, 64), np.int8))
    assert rc == 0 and np.all(Cm == 64)
    assert ctx.launches() > before
    w.free()


@pytest.mark.parametrize("K,N", [(288, 192), (2048, 1024), (6144, 2048)])
def test_tensor_core_and_gemv_routes_agree_i8(ctx, K, N):
    """Both kernel paths forced over M values that straddle the router's threshold and the 128-row tile
    (K and N tails included), each compared with the oracle."""
    L = ork_b200.lib()
    rng = np.random.default_rng(K + N)
    B = rand_i8(rng, (K, N))
    w = ctx.i8_pack(B)
    try:
        for M in (1, 7, 8, 9, 16, 24, 40, 64, 65, 100, 128, 130, 256, 512):
            A = rand_i8(rng, (M, K))
            ref = of.gemm_i32(A, B)
            for route in (1, 0):
                assert L.ork_b200_force_route(ctx.ctx, route) == 0
                rc, Cm = ctx.run(w, A)
                assert rc == 0 and np.array_equal(Cm, ref), (M, route)
    finally:
        L.ork_b200_force_route(ctx.ctx, -1)
        w.free()


@pytest.mark.parametrize("K,N", [(288, 48), (2048, 6144)])
def test_tensor_core_route_f16(ctx, K, N):
    L = ork_b200.lib()
    rng = np.random.default_rng(K * N)
    B = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    w = ctx.f16_pack(B)
    try:
        for M in (1, 16, 33, 64, 200):
            A = rng.uniform(-1, 1, size=(M, K)).astype(np.float16)
            ref = of.gemm_f16(A, B)
            for route in (1, 0):
                assert L.ork_b200_force_route(ctx.ctx, route) == 0
                rc, Cm = ctx.run(w, A)
                assert rc == 0 and np.abs(Cm - ref).max() <= f16_tol(A, B), (M, route)
    finally:
        L.ork_b200_force_route(ctx.ctx, -1)
        w.free()


@pytest.mark.parametrize("nf4", [False, True])
@pytest.mark.parametrize("K,N", [(288, 192), (2048, 1024)])
def test_tensor_core_and_gemv_routes_agree_int4(ctx, env_clean, nf4, K, N):
    """Nibble weights through both paths (the tensor-core one expands nibbles to int8 in shared memory)."""
    if nf4:
        env_clean.setenv("ORK_NF4", "1")
    L = ork_b200.lib()
    rng = np.random.default_rng(K + N + nf4)
    f32 = rng.standard_normal((N, K), dtype=np.float32)
    w, _ = ctx.i4a8_pack(f32)
    codes, _, _ = of.i4a8_blob_codes(w.dump(), K, N)
    try:
        for M in (1, 5, 16, 24, 40, 64, 65, 128, 130):
            A = rand_i8(rng, (M, K))
            ref = of.gemm_i32(A, codes)
            for route in (1, 0):
                assert L.ork_b200_force_route(ctx.ctx, route) == 0
                rc, Cm = ctx.run(w, A)
                assert rc == 0 and np.array_equal(Cm, ref), (M, route)
    finally:
        L.ork_b200_force_route(ctx.ctx, -1)
        w.free()


@pytest.mark.parametrize("na,tn,sk,flags", [(1, 128, 1, 1), (1, 128, 4, 1), (1, 128, 4, 0), (1, 128, 8, 1),
                                            (2, 128, 1, 1), (2, 128, 2, 1), (2, 128, 4, 1), (2, 128, 2, 0),
                                            (1, 256, 1, 1), (1, 256, 2, 1), (1, 192, 1, 1), (1, 192, 4, 1),
                                            (1, 192, 3, 0), (1, 64, 1, 1), (1, 64, 4, 1), (1, 64, 6, 0)])
def test_tensor_core_tile_variants_exact(ctx, env_clean, tune, na, tn, sk, flags):
    """Every non-swapped tile shape and split the router may pick (forced through its tuning variables),
    over M / N / K tails, int8 and NF4 weights; integer split-K with its zeroing ordered by the tile
    flags (default) and by a cluster barrier (flags off)."""
    tune("ORKB_TC_NA", str(na))
    tune("ORKB_TC_TN", str(tn))
    tune("ORKB_TC_SK", str(sk))
    tune("ORKB_TC_FLAGS", str(flags))
    L = ork_b200.lib()
    rng = np.random.default_rng(na * 100 + tn + sk)
    K, N = 1056, 640
    B = rand_i8(rng, (K, N))
    w8 = ctx.i8_pack(B)
    f32 = rng.standard_normal((N, K), dtype=np.float32)
    env_clean.setenv("ORK_NF4", "1")
    w4, _ = ctx.i4a8_pack(f32)
    codes, _, _ = of.i4a8_blob_codes(w4.dump(), K, N)
    try:
        assert L.ork_b200_force_route(ctx.ctx, 1) == 0
        for M in (65, 200, 256, 300, 512):
            A = rand_i8(rng, (M, K))
            rc, Cm = ctx.run(w8, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, B)), ("i8", M)
            rc, Cm = ctx.run(w4, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, codes)), ("nf4", M)
    finally:
        L.ork_b200_force_route(ctx.ctx, -1)
        w8.free()
        w4.free()


@pytest.mark.parametrize("nf4", [False, True])
@pytest.mark.parametrize("sk", [1, 3, 16])
@pytest.mark.parametrize("stages", [0, 2])
def test_tensor_core_nibble_long_k_exact(ctx, env_clean, tune, nf4, sk, stages):
    """Decode-sized M on nibble weights through the tensor-core kernel with a long K per CTA (split
    forced to 1 or 3), so the stage ring (default depth, or the 2-stage ring) wraps many times and every
    stage is expanded from nibbles; a K tail (K % 128 != 0) ends the last block. Split 16 (more than a
    cluster holds) orders its zeroing through the tile flags."""
    tune("ORKB_TC_SK", str(sk))
    if stages:
        tune("ORKB_TC_STAGES", str(stages))
    if nf4:
        env_clean.setenv("ORK_NF4", "1")
    L = ork_b200.lib()
    rng = np.random.default_rng(700 + 10 * sk + nf4)
    K, N = 4128, 384
    f32 = rng.standard_normal((N, K), dtype=np.float32)
    w, _ = ctx.i4a8_pack(f32)
    codes, _, _ = of.i4a8_blob_codes(w.dump(), K, N)
    try:
        assert L.ork_b200_force_route(ctx.ctx, 1) == 0
        for M in (1, 8, 16, 17, 32, 33, 64):
            A = rand_i8(rng, (M, K))
            rc, Cm = ctx.run(w, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, codes)), M
    finally:
        L.ork_b200_force_route(ctx.ctx, -1)
        w.free()


@pytest.mark.parametrize("sk", [12, 16])
def test_tensor_core_swapped_int8_split_past_cluster_exact(ctx, env_clean, tune, sk):
    """int8 weights at decode-sized M with a split of more than 8 (swapped tiles, tile flags), M and K
    tails."""
    tune("ORKB_TC_SK", str(sk))
    L = ork_b200.lib()
    rng = np.random.default_rng(900 + sk)
    K, N = 8224, 384
    B = rand_i8(rng, (K, N))
    w = ctx.i8_pack(B)
    try:
        assert L.ork_b200_force_route(ctx.ctx, 1) == 0
        for M in (1, 8, 13, 40):
            A = rand_i8(rng, (M, K))
            rc, Cm = ctx.run(w, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, B)), M
    finally:
        L.ork_b200_force_route(ctx.ctx, -1)
        w.free()


@pytest.mark.parametrize("nf4", [False, True])
def test_tensor_core_nibble_wide_grid_exact(ctx, env_clean, nf4):
    """Nibble weights wide enough (N > 296 * 128) that the router picks the 2-stage ring with a 2-way
    split for M <= 16, through the default choice (no tuning variables), with a K tail."""
    if nf4:
        env_clean.setenv("ORK_NF4", "1")
    L = ork_b200.lib()
    rng = np.random.default_rng(800 + nf4)
    K, N = 1056, 297 * 128
    f32 = rng.standard_normal((N, K), dtype=np.float32)
    w, _ = ctx.i4a8_pack(f32)
    codes, _, _ = of.i4a8_blob_codes(w.dump(), K, N)
    try:
        assert L.ork_b200_force_route(ctx.ctx, 1) == 0
        for M in (1, 8, 16):
            A = rand_i8(rng, (M, K))
            rc, Cm = ctx.run(w, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, codes)), M
    finally:
        L.ork_b200_force_route(ctx.ctx, -1)
        w.free()


@pytest.mark.parametrize("pair,tn,sk,flags", [(2, 256, 1, 1), (2, 256, 2, 1), (2, 256, 4, 1), (2, 256, 2, 0),
                                              (2, 128, 1, 1), (2, 128, 4, 1), (2, 64, 1, 1), (2, 64, 2, 1),
                                              (2, 192, 1, 1), (2, 192, 4, 1), (2, 192, 3, 0), (3, 0, 1, 1),
                                              (3, 0, 2, 1), (3, 0, 4, 1), (3, 0, 4, 0)])
def test_tensor_core_pair_tiles_exact(ctx, env_clean, tune, pair, tn, sk, flags):
    """CTA-pair (cta_group::2) tiles forced through the tuning variables: pair = 2 puts the activations
    on the 256-row side (M tails leave the second CTA of the last pair entirely out of range at
    M = 300), pair = 3 the weight (N tails, narrow M). int8, NF4 and uniform int4 exact; f16 within
    its tolerance. Integer split-K through the tile flags (default) and through the cluster barrier."""
    tune("ORKB_TC_PAIR", str(pair))
    if tn:
        tune("ORKB_TC_TN", str(tn))
    tune("ORKB_TC_SK", str(sk))
    tune("ORKB_TC_FLAGS", str(flags))
    L = ork_b200.lib()
    rng = np.random.default_rng(pair * 1000 + tn + sk)
    K, N = 1056, 640
    B = rand_i8(rng, (K, N))
    w8 = ctx.i8_pack(B)
    f32 = rng.standard_normal((N, K), dtype=np.float32)
    env_clean.setenv("ORK_NF4", "1")
    wn, _ = ctx.i4a8_pack(f32)
    env_clean.delenv("ORK_NF4")
    wu, _ = ctx.i4a8_pack(f32)
    cn, _, _ = of.i4a8_blob_codes(wn.dump(), K, N)
    cu, _, _ = of.i4a8_blob_codes(wu.dump(), K, N)
    Bh = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    wh = ctx.f16_pack(Bh)
    Ms = (65, 200, 256, 300, 512, 700) if pair == 2 else (40, 100, 128, 200, 256)
    try:
        assert L.ork_b200_force_route(ctx.ctx, 1) == 0
        for M in Ms:
            A = rand_i8(rng, (M, K))
            rc, Cm = ctx.run(w8, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, B)), ("i8", M)
            rc, Cm = ctx.run(wn, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, cn)), ("nf4", M)
            rc, Cm = ctx.run(wu, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, cu)), ("u4", M)
            Ah = rng.uniform(-1, 1, size=(M, K)).astype(np.float16)
            rc, Cm = ctx.run(wh, Ah)
            assert rc == 0 and np.abs(Cm - of.gemm_f16(Ah, Bh)).max() <= f16_tol(Ah, Bh), ("f16", M)
    finally:
        L.ork_b200_force_route(ctx.ctx, -1)
        for w in (w8, wn, wu, wh):
            w.free()


@pytest.mark.parametrize("kind,cpw", [("staged", 0), ("direct", 1), ("direct", 2), ("direct", 4)])
def test_decode_kernels_exact_all_formats(ctx, env_clean, tune, kind, cpw):
    """Both decode kernels, forced through the tuning variables, on every weight format and M = 1..8,
    including a row far beyond the staged kernel's shared memory (K = 24576: always the direct kernel)."""
    L = ork_b200.lib()
    if kind == "direct":
        tune("ORKB_GEMV_KIND", "1")
        tune("ORKB_GEMV_CPW", str(cpw))
    else:
        tune("ORKB_GEMV_KIND", "0")
    rng = np.random.default_rng(cpw + 40)
    try:
        assert L.ork_b200_force_route(ctx.ctx, 0) == 0
        for K, N in ((2048, 96), (24576, 64)):
            B = rand_i8(rng, (K, N))
            f32 = rng.standard_normal((N, K), dtype=np.float32)
            w8 = ctx.i8_pack(B)
            wu, _ = ctx.i4a8_pack(f32)
            env_clean.setenv("ORK_NF4", "1")
            wn, _ = ctx.i4a8_pack(f32)
            env_clean.delenv("ORK_NF4")
            cu, _, _ = of.i4a8_blob_codes(wu.dump(), K, N)
            cn, _, _ = of.i4a8_blob_codes(wn.dump(), K, N)
            Bh = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
            wh = ctx.f16_pack(Bh)
            try:
                for M in (1, 2, 3, 5, 8, 11):
                    A = rand_i8(rng, (M, K))
                    for w, codes, tag in ((w8, B, "i8"), (wu, cu, "u4"), (wn, cn, "nf4")):
                        rc, Cm = ctx.run(w, A)
                        assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, codes)), (tag, K, M)
                    Ah = rng.uniform(-1, 1, size=(M, K)).astype(np.float16)
                    rc, Cm = ctx.run(wh, Ah)
                    assert rc == 0 and np.abs(Cm - of.gemm_f16(Ah, Bh)).max() <= f16_tol(Ah, Bh), ("f16", K, M)
            finally:
                for w in (w8, wu, wn, wh):
                    w.free()
    finally:
        L.ork_b200_force_route(ctx.ctx, -1)
