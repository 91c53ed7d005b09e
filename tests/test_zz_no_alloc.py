"""ork_i8_mm_run_noalloc against ork_i8_mm_run, through the C ABI (needs a B200).

The no-allocation entry point serves callers that cannot let a library allocate device memory at run
time (an engine that reserved nearly all HBM for its own pool, a hard device-memory cap, or code that
must not trigger cudaMalloc's device-wide synchronisation). It stages A and C through a fixed 4 MiB
scratch area built into the library instead of context-allocated buffers, so its results must equal
the regular entry point's exactly (int32), call after call, while the scratch keeps the previous call's
contents. This file is collected last so that, if it fails, every other test has already run; it also
passes alone in a fresh process (it builds its own weights on the session context).
"""
import numpy as np
import pytest

import oracle_ffi as of
import ork_b200

pytestmark = pytest.mark.gpu


def _noalloc(ctx, w, A):
    M = A.shape[0]
    Cm = np.full((M, w.N), -7, np.int32)
    rc = ork_b200.lib().ork_i8_mm_run_noalloc(ctx.ctx, w.h, M, A.ctypes.data, Cm.ctypes.data)
    return rc, Cm


# M = 1 and 4 take the CUDA-core GEMV, 16 and 128 the tensor-core kernel
@pytest.mark.parametrize("K,N,M", [(2048, 2048, 1), (2048, 6144, 4), (6144, 2048, 16), (2048, 2048, 128)])
def test_noalloc_equals_regular_entry_point_twice(ctx, K, N, M):
    rng = np.random.default_rng(K + N + M)
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    w = ctx.i8_pack(B)
    try:
        for call in range(2):  # the second call runs over the first call's leftovers in the scratch
            A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
            rc_ref, ref = ctx.run(w, A)
            rc, got = _noalloc(ctx, w, A)
            assert rc_ref == 0 and rc == 0, call
            assert np.array_equal(got, ref), call
            assert np.array_equal(got, of.gemm_i32(A, B)), call
    finally:
        w.free()


def test_noalloc_int4_store_twice(ctx, env_clean):
    env_clean.setenv("ORK_NF4", "1")
    K, N = 2048, 512
    rng = np.random.default_rng(5)
    f32 = rng.standard_normal((N, K), dtype=np.float32)
    w, _ = ctx.i4a8_pack(f32)
    try:
        for M in (1, 40):
            A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
            rc_ref, ref = ctx.run(w, A)
            rc, got = _noalloc(ctx, w, A)
            assert rc_ref == 0 and rc == 0 and np.array_equal(got, ref), M
    finally:
        w.free()


def test_noalloc_refuses_what_does_not_fit(ctx):
    K, N, M = 2048, 2048, 512  # 1 MiB of A + 4 MiB of C > 4 MiB
    w = ctx.i8_pack(np.ones((K, N), np.int8))
    try:
        rc, _ = _noalloc(ctx, w, np.ones((M, K), np.int8))
        assert rc == -1
        rc, got = _noalloc(ctx, w, np.ones((8, K), np.int8))  # still usable afterwards
        assert rc == 0 and np.all(got == K)
    finally:
        w.free()


def test_noalloc_refuses_bad_arguments(ctx):
    L = ork_b200.lib()
    w = ctx.i4_pack(np.zeros((64, 64), np.int8))  # W4A4 weights belong to ork_i4_mm_run
    A = np.zeros((1, 64), np.int8)
    Cm = np.zeros((1, 64), np.int32)
    try:
        assert L.ork_i8_mm_run_noalloc(ctx.ctx, w.h, 1, A.ctypes.data, Cm.ctypes.data) == -1
        assert L.ork_i8_mm_run_noalloc(None, w.h, 1, A.ctypes.data, Cm.ctypes.data) == -1
        shared = np.zeros(512, np.int8)
        w8 = ctx.i8_pack(np.ones((64, 64), np.int8))
        assert L.ork_i8_mm_run_noalloc(ctx.ctx, w8.h, 1, shared.ctypes.data, shared.ctypes.data + 16) == -1
        w8.free()
    finally:
        w.free()


def test_noalloc_allocates_nothing_on_a_fresh_context():
    """What the entry point exists for: on a context that has never run anything, two calls with host
    buffers leave the context without any run-time staging (ork_b200_staging_bytes stays 0), while one
    ork_i8_mm_run on the same context does allocate its staging buffers."""
    L = ork_b200.lib()
    K, N, M = 2048, 1024, 8
    rng = np.random.default_rng(17)
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    with ork_b200.Context() as fresh:
        w = fresh.i8_pack(B)
        try:
            assert L.ork_b200_staging_bytes(fresh.ctx) == 0
            for call in range(2):
                A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
                rc, got = _noalloc(fresh, w, A)
                assert rc == 0 and np.array_equal(got, of.gemm_i32(A, B)), call
                assert L.ork_b200_staging_bytes(fresh.ctx) == 0, call
            rc, _ = fresh.run(w, A)
            assert rc == 0 and L.ork_b200_staging_bytes(fresh.ctx) > 0
        finally:
            w.free()


def test_noalloc_device_buffers_in_place_beyond_the_scratch(ctx):
    """Device-resident A and C are used in place, as by ork_i8_mm_run, so a run whose host buffers would
    not fit the 4 MiB scratch (1 MiB of A + 4 MiB of C) works when they are device memory."""
    import torch

    L = ork_b200.lib()
    K, N, M = 2048, 2048, 512
    rng = np.random.default_rng(23)
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    w = ctx.i8_pack(B)
    try:
        A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
        dA = torch.from_numpy(A).cuda()
        dC = torch.zeros((M, N), dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        assert L.ork_i8_mm_run_noalloc(ctx.ctx, w.h, M, dA.data_ptr(), dC.data_ptr()) == 0
        assert np.array_equal(dC.cpu().numpy(), of.gemm_i32(A, B))
    finally:
        w.free()
