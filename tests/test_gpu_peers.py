"""Column-sharded runs with the output gather fused into the matmul over peer memory (ork_b200_peers_*,
ork_b200_i8_mm_run_peers_async / ork_b200_i4_mm_run_peers_async, and the one-call run + gather
ork_b200_i8_mm_run_gather_async / ork_b200_i4_mm_run_gather_async, include/ork_b200.h).

Output channels are independent (ork-driver src/npu/i4/pack.c:63-80), so rank g packs channels
[g*N/R, (g+1)*N/R) and its run writes them into every rank's C; after ork_b200_peers_wait_async each
rank's C must equal the unsharded oracle product exactly. One-rank tables run on any GPU; the two-rank
test needs two GPUs (one process each) and is skipped otherwise. The bounded wait is tested on one rank
with a flag that nothing sets (no GPU fault: the wait gives up and the next sync reports it).
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest

import oracle_ffi as of
import ork_b200

pytestmark = pytest.mark.gpu
_p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731


class _NoDist:
    @staticmethod
    def is_initialized():
        return False


def _read(ctx, ptr, shape):
    out = np.empty(shape, np.int32)
    assert ctx.L.ork_b200_copy(ctx.ctx, _p(out), ptr, out.nbytes) == 0
    return out


def test_one_rank_table(ctx):
    import torch

    import shard

    L = ctx.L
    dev = torch.device("cuda", L.ork_b200_device(ctx.ctx))
    rng = np.random.default_rng(41)
    K, N, Mmax = 1024, 256, 40
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    w = ctx.i8_pack(B)
    g = shard.PeerGroup(ctx, _NoDist)
    t, cptr = g.table(Mmax, N, N)
    for M in (1, 5, 8, 40):  # decode and tensor-core matmuls; run + wait, then the one-call run + gather
        A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
        tA = torch.from_numpy(A).to(dev)
        torch.cuda.synchronize()
        assert L.ork_b200_i8_mm_run_peers_async(ctx.ctx, w.h, M, tA.data_ptr(), t) == 0
        assert L.ork_b200_peers_wait_async(ctx.ctx, t) == 0
        assert L.ork_b200_sync(ctx.ctx) == 0
        assert np.array_equal(_read(ctx, cptr, (M, N)), of.gemm_i32(A, B)), M
        A2 = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
        tA = torch.from_numpy(A2).to(dev)
        torch.cuda.synchronize()
        assert L.ork_b200_i8_mm_run_gather_async(ctx.ctx, w.h, M, tA.data_ptr(), t) == 0
        assert L.ork_b200_sync(ctx.ctx) == 0
        assert np.array_equal(_read(ctx, cptr, (M, N)), of.gemm_i32(A2, B)), M
    # the tagged-word gather (landing buffers attached for up to Mmax rows)
    tl, cl = g.table(Mmax, N, N, land=True)
    for M in (1, 8, 40):
        A3 = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
        tA = torch.from_numpy(A3).to(dev)
        torch.cuda.synchronize()
        assert L.ork_b200_i8_mm_run_gather_async(ctx.ctx, w.h, M, tA.data_ptr(), tl) == 0
        assert L.ork_b200_sync(ctx.ctx) == 0
        assert np.array_equal(_read(ctx, cl, (M, N)), of.gemm_i32(A3, B)), ("tagged", M)
    w.free()
    g.close()


def test_wait_without_signal_gives_up(ctx):
    """A two-rank table whose second rank is a buffer of this process that no run ever signals from: the
    run posts its signals, the wait for the missing rank's gives up (bounded, ~2 s), the next sync reports
    it once and the context keeps working -- through the separate wait and through the one-call gather."""
    import torch

    L = ctx.L
    dev = torch.device("cuda", L.ork_b200_device(ctx.ctx))
    K, N = 256, 64
    rng = np.random.default_rng(5)
    B = rng.integers(-128, 128, size=(K, N // 2), dtype=np.int8)
    w = ctx.i8_pack(B)
    h = (C.c_uint8 * 64)()
    bufs = [L.ork_b200_sym_alloc(ctx.ctx, N * 4, h) for _ in range(2)]
    flags = [L.ork_b200_sym_alloc(ctx.ctx, 64, h) for _ in range(2)]
    assert all(bufs) and all(flags)
    arr = C.c_void_p * 2
    t = L.ork_b200_peers_create(ctx.ctx, 2, 0, arr(*bufs), arr(*flags), N, 0, N // 2)
    assert t
    tA = torch.from_numpy(rng.integers(-128, 128, size=(1, K), dtype=np.int8)).to(dev)
    torch.cuda.synchronize()
    try:
        assert L.ork_b200_i8_mm_run_peers_async(ctx.ctx, w.h, 1, tA.data_ptr(), t) == 0
        assert L.ork_b200_peers_wait_async(ctx.ctx, t) == 0  # rank 1 never signals
        assert L.ork_b200_sync(ctx.ctx) == -1
        assert L.ork_b200_sync(ctx.ctx) == 0  # the flag was cleared; the context keeps working
        assert L.ork_b200_i8_mm_run_gather_async(ctx.ctx, w.h, 1, tA.data_ptr(), t) == 0
        assert L.ork_b200_sync(ctx.ctx) == -1
        assert L.ork_b200_sync(ctx.ctx) == 0
        # this rank's own columns did arrive in its C
        assert np.array_equal(_read(ctx, bufs[0], (1, N))[:, : N // 2], of.gemm_i32(tA.cpu().numpy(), B))
    finally:
        L.ork_b200_peers_destroy(t)
        for p in bufs + flags:
            L.ork_b200_sym_free(ctx.ctx, p)
        w.free()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _two_rank_worker(rank, world, port, kind):
    import datetime

    import torch
    import torch.distributed as dist

    import shard

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    ctx = ork_b200.Context()
    L = ctx.L
    dev = torch.device("cuda", rank)
    rng = np.random.default_rng(77)  # the same full weight and activations on every rank
    K, N, Mmax = 2048, 512, 24
    ncols = N // world
    n0 = rank * ncols
    if kind == "i8":
        B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
        w = ctx.i8_pack(np.ascontiguousarray(B[:, n0:n0 + ncols]))
        run, gather = L.ork_b200_i8_mm_run_peers_async, L.ork_b200_i8_mm_run_gather_async
    else:
        B = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
        w = ctx.i4_pack(np.ascontiguousarray(B[:, n0:n0 + ncols]))
        run, gather = L.ork_b200_i4_mm_run_peers_async, L.ork_b200_i4_mm_run_gather_async
    g = shard.PeerGroup(ctx, dist)
    t, cptr = g.table(Mmax, N, ncols)
    t2, cptr2 = g.table(Mmax, N, ncols)
    tl = [g.table(Mmax, N, ncols, land=True) for _ in range(2)]  # tagged-word gather tables
    try:
        for M in (1, 8, 3, 24):
            A = rng.integers(-128 if kind == "i8" else -8, 128 if kind == "i8" else 8, size=(M, K), dtype=np.int8)
            tA = torch.from_numpy(A).to(dev)
            torch.cuda.synchronize()
            assert run(ctx.ctx, w.h, M, tA.data_ptr(), t) == 0
            assert L.ork_b200_peers_wait_async(ctx.ctx, t) == 0
            assert L.ork_b200_sync(ctx.ctx) == 0
            assert np.array_equal(_read(ctx, cptr, (M, N)), of.gemm_i32(A, B)), (rank, M)
            dist.barrier()  # every rank has read C before anyone runs again (the buffers' reuse rule)
            # the same through the one-call run + gather (its push kernel waits for every rank's signal)
            A = rng.integers(-128 if kind == "i8" else -8, 128 if kind == "i8" else 8, size=(M, K), dtype=np.int8)
            tA = torch.from_numpy(A).to(dev)
            torch.cuda.synchronize()
            assert gather(ctx.ctx, w.h, M, tA.data_ptr(), t) == 0
            assert L.ork_b200_sync(ctx.ctx) == 0
            assert np.array_equal(_read(ctx, cptr, (M, N)), of.gemm_i32(A, B)), (rank, M, "gather")
            dist.barrier()
            # and through the tagged-word gather (landing buffers), alternating its two tables
            A = rng.integers(-128 if kind == "i8" else -8, 128 if kind == "i8" else 8, size=(M, K), dtype=np.int8)
            tA = torch.from_numpy(A).to(dev)
            torch.cuda.synchronize()
            tt, tc = tl[M % 2]
            assert gather(ctx.ctx, w.h, M, tA.data_ptr(), tt) == 0
            assert L.ork_b200_sync(ctx.ctx) == 0
            assert np.array_equal(_read(ctx, tc, (M, N)), of.gemm_i32(A, B)), (rank, M, "tagged")
            dist.barrier()
        # the run + wait pair captured once and replayed: the counts advance on the device
        M = 4
        A = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
        tA = torch.from_numpy(A).to(dev)
        s = torch.cuda.ExternalStream(L.ork_b200_stream(ctx.ctx))
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            assert run(ctx.ctx, w.h, M, tA.data_ptr(), t) == 0
            assert L.ork_b200_peers_wait_async(ctx.ctx, t) == 0
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            assert L.ork_b200_sync(ctx.ctx) == 0
            assert np.array_equal(_read(ctx, cptr, (M, N)), of.gemm_i32(A, B))
            dist.barrier()
        del graph
        # a captured chain of tagged gathers alternating two tables, replayed (the tags advance on the device)
        A = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
        tA = torch.from_numpy(A).to(dev)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for i in range(4):
                assert gather(ctx.ctx, w.h, M, tA.data_ptr(), tl[i % 2][0]) == 0
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            assert L.ork_b200_sync(ctx.ctx) == 0
            for _, tc in tl:
                assert np.array_equal(_read(ctx, tc, (M, N)), of.gemm_i32(A, B)), "tagged graph"
            dist.barrier()
        del graph
        # a captured chain of run + gather calls alternating between two tables (the reuse rule), replayed
        A = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
        tA = torch.from_numpy(A).to(dev)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for i in range(4):
                assert gather(ctx.ctx, w.h, M, tA.data_ptr(), t if i % 2 == 0 else t2) == 0
        for _ in range(3):
            graph.replay()
            torch.cuda.synchronize()
            assert L.ork_b200_sync(ctx.ctx) == 0
            assert np.array_equal(_read(ctx, cptr, (M, N)), of.gemm_i32(A, B))
            assert np.array_equal(_read(ctx, cptr2, (M, N)), of.gemm_i32(A, B))
            dist.barrier()
        del graph
    finally:
        g.close()
        w.free()
        ctx.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("kind", ["i8", "i4"])
def test_two_ranks_fused_gather(kind):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_two_rank_worker, args=(2, _free_port(), kind), nprocs=2, join=True)


def test_two_devices_one_process():
    """Contexts on two GPUs of one process: every kernel's shared-memory opt-in and the error word are set
    per device, so the tensor-core, decode and fused-output paths all run exactly on the second GPU too."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    rng = np.random.default_rng(91)
    K, N = 2048, 512
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    ctxs = []
    try:
        for dev in (0, 1):
            torch.cuda.set_device(dev)
            ctxs.append(ork_b200.Context())
        for ctx in ctxs:
            w = ctx.i8_pack(B)
            for M in (1, 8, 300):
                A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
                rc, Cm = ctx.run(w, A)
                assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, B)), M
                c8 = np.zeros((M, N), np.int8)
                assert ctx.L.ork_i8_mm_run_out8(ctx.ctx, w.h, M, _p(A), _p(c8), 0x1000, 15) == 0
                assert np.array_equal(c8, of.requant(of.gemm_i32(A, B), 0x1000, 15)), M
            w.free()
    finally:
        for ctx in ctxs:
            ctx.close()
        torch.cuda.set_device(0)
