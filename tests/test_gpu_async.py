"""The reference's asynchronous run API (ork_*_mm_run_async / ork_async_wait, include/ork/chain.h:124-143)
and the device-pointer checks of the B200 stream-ordered entry points (needs a B200).

ork_async jobs over pageable host memory, pinned host memory and device memory must give the same C
as the synchronous call (bit-exact int32 against the oracle; fp16 within the north-star tolerance); one
job may be in flight per context, and every other run on it is refused until the wait. The
device-pointer entry points (include/ork_b200.h) must refuse host buffers with -1 (-3 for the layer
calls) before launching anything.
"""
import ctypes as C

import numpy as np
import pytest

import oracle_ffi as of
import ork_b200
from ork_b200 import TaskI4, TaskI8

pytestmark = pytest.mark.gpu


def _p(a):
    return C.c_void_p(a.ctypes.data)


def f16_tol(A, B):
    K = A.shape[1]
    return 1e-3 * np.sqrt(K) * float(np.abs(A.astype(np.float32)).max()) * float(np.abs(B.astype(np.float32)).max())


@pytest.mark.parametrize("mem", ["pageable", "pinned", "device"])
@pytest.mark.parametrize("M", [1, 8, 37, 300])
def test_i8_async_matches_oracle(ctx, mem, M):
    import torch

    L = ork_b200.lib()
    rng = np.random.default_rng(M * 3 + len(mem))
    K, N = 2048, 1536
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    w = ctx.i8_pack(B)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    ref = of.gemm_i32(A, B)
    try:
        if mem == "device":
            tA = torch.from_numpy(A).cuda()
            tC = torch.zeros((M, N), dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            h = L.ork_i8_mm_run_async(ctx.ctx, w.h, M, tA.data_ptr(), tC.data_ptr())
            assert h
            assert L.ork_async_wait(h) == 0
            assert np.array_equal(tC.cpu().numpy(), ref)
            return
        if mem == "pinned":
            tA = torch.from_numpy(A).pin_memory()
            tC = torch.zeros((M, N), dtype=torch.int32).pin_memory()
            pa, pc = tA.data_ptr(), tC.data_ptr()
            out = tC.numpy()
        else:
            out = np.full((M, N), -7, np.int32)
            pa, pc = A.ctypes.data, out.ctypes.data
        h = L.ork_i8_mm_run_async(ctx.ctx, w.h, M, pa, pc)
        assert h
        assert L.ork_async_wait(h) == 0
        assert np.array_equal(out, ref)
        assert L.ork_npu_last_async_cpu(ctx.ctx) >= 0
    finally:
        w.free()


def test_f16_and_i4_async(ctx):
    L = ork_b200.lib()
    rng = np.random.default_rng(5)
    K, N, M = 1024, 768, 24
    Bh = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    wh = ctx.f16_pack(Bh)
    Ah = rng.uniform(-1, 1, size=(M, K)).astype(np.float16)
    Ch = np.zeros((M, N), np.float32)
    B4 = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    w4 = ctx.i4_pack(B4)
    A4 = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
    C4 = np.zeros((M, N), np.int32)
    try:
        h = L.ork_mm_run_async(ctx.ctx, wh.h, M, _p(Ah), _p(Ch))
        assert h and L.ork_async_wait(h) == 0
        assert np.abs(Ch - of.gemm_f16(Ah, Bh)).max() <= f16_tol(Ah, Bh)
        h = L.ork_i4_mm_run_async(ctx.ctx, w4.h, M, _p(A4), _p(C4))
        assert h and L.ork_async_wait(h) == 0
        assert np.array_equal(C4, of.gemm_i32(A4, B4))
        # the reference's worker reports a dtype mismatch through the wait; here the queueing does
        h = L.ork_mm_run_async(ctx.ctx, w4.h, M, _p(Ah), _p(Ch))
        assert h and L.ork_async_wait(h) == -1
        # int8 launcher on a non-int8 weight: NULL (src/npu/i8/run.c:779)
        assert not L.ork_i8_mm_run_async(ctx.ctx, w4.h, M, _p(A4), _p(C4))
    finally:
        wh.free()
        w4.free()


@pytest.mark.parametrize("kind", ["chain", "stream"])
def test_batch_async_with_strided_c(ctx, kind):
    """S independent int8 matmuls (decode-sized and larger) writing into one strided host C, and a W4A4
    batch, through the _chain_async / _stream_async launchers."""
    L = ork_b200.lib()
    rng = np.random.default_rng(11 if kind == "chain" else 12)
    K = 1024
    Ns = [256, 512, 320]
    Ms = [1, 5, 40]
    Bs = [rng.integers(-128, 128, size=(K, n), dtype=np.int8) for n in Ns]
    ws = [ctx.i8_pack(b) for b in Bs]
    As = [rng.integers(-128, 128, size=(m, K), dtype=np.int8) for m in Ms]
    width = sum(Ns) + 64
    Cbig = np.zeros((max(Ms), width), np.int32)
    tasks, off = [], 0
    for w, a, n in zip(ws, As, Ns):
        tasks.append(TaskI8(w.h, a.shape[0], a.ctypes.data, Cbig[:, off:].ctypes.data, width))
        off += n
    arr = (TaskI8 * len(tasks))(*tasks)
    B4 = rng.integers(-8, 8, size=(K, 128), dtype=np.int8)
    w4 = ctx.i4_pack(B4)
    A4 = [rng.integers(-8, 8, size=(m, K), dtype=np.int8) for m in (1, 9)]
    C4 = [np.zeros((a.shape[0], 128), np.int32) for a in A4]
    arr4 = (TaskI4 * 2)(*[TaskI4(w4.h, a.shape[0], a.ctypes.data, c.ctypes.data) for a, c in zip(A4, C4)])
    try:
        f8 = L.ork_i8_mm_run_chain_async if kind == "chain" else L.ork_i8_mm_run_stream_async
        f4 = L.ork_i4_mm_run_chain_async if kind == "chain" else L.ork_i4_mm_run_stream_async
        h = f8(ctx.ctx, len(tasks), arr)
        assert h and L.ork_async_wait(h) == 0
        off = 0
        for a, b, n in zip(As, Bs, Ns):
            assert np.array_equal(Cbig[:a.shape[0], off:off + n], of.gemm_i32(a, b))
            off += n
        h = f4(ctx.ctx, 2, arr4)
        assert h and L.ork_async_wait(h) == 0
        for a, c in zip(A4, C4):
            assert np.array_equal(c, of.gemm_i32(a, B4))
        for c in C4:
            c[:] = 0
        assert L.ork_i4_mm_run_stream(ctx.ctx, 2, arr4) == 0
        for a, c in zip(A4, C4):
            assert np.array_equal(c, of.gemm_i32(a, B4))
    finally:
        for w in ws + [w4]:
            w.free()


def test_one_job_in_flight(ctx):
    """While a job is in flight a second launch returns NULL and every other run on the context is refused
    (-1) without touching its C; after the wait both work again."""
    L = ork_b200.lib()
    rng = np.random.default_rng(3)
    K, N, M = 4096, 4096, 64
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    w = ctx.i8_pack(B)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    C1 = np.zeros((M, N), np.int32)
    C2 = np.full((M, N), 5, np.int32)
    try:
        h = L.ork_i8_mm_run_async(ctx.ctx, w.h, M, _p(A), _p(C1))
        assert h
        assert not L.ork_i8_mm_run_async(ctx.ctx, w.h, M, _p(A), _p(C2))
        assert L.ork_i8_mm_run(ctx.ctx, w.h, M, _p(A), _p(C2)) == -1
        assert L.ork_mm_submit(ctx.ctx, w.h, M, _p(A)) == -1
        assert (C2 == 5).all()
        assert L.ork_async_wait(h) == 0
        ref = of.gemm_i32(A, B)
        assert np.array_equal(C1, ref)
        assert L.ork_i8_mm_run(ctx.ctx, w.h, M, _p(A), _p(C2)) == 0 and np.array_equal(C2, ref)
    finally:
        w.free()


def test_device_entry_points_refuse_host_buffers(ctx):
    """Host buffers handed to the device-pointer entry points: -1 (-3 for the layer calls), no launch."""
    import torch

    L = ork_b200.lib()
    rng = np.random.default_rng(9)
    K, N, M = 512, 128, 4
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    w = ctx.i8_pack(B)
    A = np.zeros((M, K), np.int8)
    Cm = np.zeros((M, N), np.int32)
    dA = torch.zeros((M, K), dtype=torch.int8, device="cuda")
    dC = torch.zeros((M, N), dtype=torch.int32, device="cuda")
    f = np.zeros(4096, np.float32)
    n0 = ctx.launches()
    try:
        assert L.ork_b200_i8_mm_run_async(ctx.ctx, w.h, M, _p(A), dC.data_ptr()) == -1
        assert L.ork_b200_i8_mm_run_async(ctx.ctx, w.h, M, dA.data_ptr(), _p(Cm)) == -1
        assert L.ork_b200_i8_mm_run_out8_async(ctx.ctx, w.h, M, _p(A), dC.data_ptr(), 1, 0) == -1
        arr = (TaskI8 * 1)(TaskI8(w.h, M, A.ctypes.data, Cm.ctypes.data, 0))
        assert L.ork_b200_i8_mm_run_chain_async(ctx.ctx, 1, arr) == -1
        assert L.ork_b200_rows_q8_async(ctx.ctx, _p(f), None, 1, 128, 1, dA.data_ptr(), None) == -1
        assert L.ork_b200_rows_dequant_async(ctx.ctx, _p(Cm), M, N, dC.data_ptr(), None, None, dC.data_ptr()) == -1
        assert L.ork_b200_argmax_scaled_async(ctx.ctx, dC.data_ptr(), _p(f), N, dC.data_ptr()) == -1
        assert ctx.launches() == n0
    finally:
        w.free()


@pytest.mark.parametrize("kind,K,N,M", [("i8", 2048, 2048, 512), ("i8", 6144, 2048, 300), ("i8", 1024, 8192, 40),
                                        ("i4", 2048, 4096, 200), ("f16", 1024, 4096, 96)])
def test_pinned_host_runs_in_row_blocks(ctx, kind, K, N, M):
    """A synchronous run over pinned host buffers with at least 1 MiB of results goes through in row blocks
    on three streams (upload, matmul, readback overlapping); C must equal the oracle's exactly (fp16:
    within the tolerance), row tails included, and equal the one-piece result of pageable buffers."""
    import torch

    L = ork_b200.lib()
    rng = np.random.default_rng(K + N + M)
    if kind == "f16":
        B = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
        w = ctx.f16_pack(B)
        A = rng.uniform(-1, 1, size=(M, K)).astype(np.float16)
        tA, tC = torch.from_numpy(A).pin_memory(), torch.zeros((M, N), dtype=torch.float32).pin_memory()
        fn = L.ork_f16_mm_run
    else:
        lo, hi = (-8, 8) if kind == "i4" else (-128, 128)
        B = rng.integers(lo, hi, size=(K, N), dtype=np.int8)
        w = ctx.i4_pack(B) if kind == "i4" else ctx.i8_pack(B)
        A = rng.integers(lo, hi, size=(M, K), dtype=np.int8)
        tA, tC = torch.from_numpy(A).pin_memory(), torch.zeros((M, N), dtype=torch.int32).pin_memory()
        fn = L.ork_i4_mm_run if kind == "i4" else L.ork_i8_mm_run
    try:
        for _ in range(2):
            tC.zero_()
            assert fn(ctx.ctx, w.h, M, tA.data_ptr(), tC.data_ptr()) == 0
            got = tC.numpy()
            rc, one_piece = ctx.run(w, A)
            assert rc == 0
            if kind == "f16":
                assert np.abs(got - of.gemm_f16(A, B)).max() <= f16_tol(A, B)
            else:
                assert np.array_equal(got, of.gemm_i32(A, B))
                assert np.array_equal(got, one_piece)
    finally:
        w.free()
