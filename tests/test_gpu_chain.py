"""Batches of independent matmuls (ork_i8_mm_run_chain / _stream / _chain_async, ork_i4_mm_run_chain /
_experts) and the ork_mm_submit / ork_mm_collect ring, through the C ABI.

The reference's offline meaning of a batch is every task computed exactly on its own
(src/npu/core/buf.c:560-564): each task's C must equal the oracle's int32 product, whatever mix of
formats, M, host or device buffers and C row strides the batch holds, and the bytes between strided C
rows must stay untouched. Decode-sized tasks of one format share one launch (checked by the launch
counter); larger tasks take the ordinary route.
"""
import ctypes as C

import numpy as np
import pytest

import oracle_ffi as of
import ork_b200
from ork_b200 import TaskI4, TaskI8

pytestmark = pytest.mark.gpu
_p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731


def _weights(ctx, env, rng, shapes):
    """(weight, codes [K][N]) for int8, uniform int4 and NF4 stores of each (K, N)."""
    out = []
    for i, (K, N) in enumerate(shapes):
        kind = i % 3
        if kind == 0:
            B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
            out.append((ctx.i8_pack(B), B))
        else:
            if kind == 2:
                env.setenv("ORK_NF4", "1")
            w, _ = ctx.i4a8_pack(rng.standard_normal((N, K), dtype=np.float32))
            env.delenv("ORK_NF4", raising=False)
            codes, _, _ = of.i4a8_blob_codes(w.dump(), K, N)
            out.append((w, codes))
    return out


def test_i8_chain_mixed_batch_exact(ctx, env_clean):
    rng = np.random.default_rng(11)
    shapes = [(256, 64), (1024, 96), (2048, 256), (512, 128), (1024, 64), (256, 192), (2048, 128), (768, 64)]
    ws = _weights(ctx, env_clean, rng, shapes)
    Ms = [1, 3, 8, 2, 40, 5, 1, 130]
    tasks, outs, pads = [], [], []
    keep = []
    for i, ((w, codes), M) in enumerate(zip(ws, Ms)):
        K, N = shapes[i]
        A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
        cs = N + (16 if i % 2 else 0)  # every other task writes into a wider C
        Cb = np.full((M, cs), -5, np.int32)
        tasks.append(TaskI8(w.h, M, A.ctypes.data, Cb.ctypes.data, cs if i % 2 else 0))
        outs.append((Cb, A, codes, N, cs))
        keep.append(A)
    arr = (TaskI8 * len(tasks))(*tasks)
    l0 = ctx.launches()
    assert ctx.L.ork_i8_mm_run_chain(ctx.ctx, len(tasks), arr) == 0
    launches = ctx.launches() - l0
    for i, (Cb, A, codes, N, cs) in enumerate(outs):
        assert np.array_equal(Cb[:, :N], of.gemm_i32(A, codes)), i
        assert np.all(Cb[:, N:] == -5), i  # the gaps of a strided C are untouched
    # decode-sized tasks: one launch per weight format (3); M=40 and M=130 take their own launches
    assert launches <= 3 + 2, launches
    for w, _ in ws:
        w.free()


def test_chain_many_experts_one_launch_per_format(ctx):
    """An MoE-like batch beyond one launch's task table (130 experts of one format)."""
    rng = np.random.default_rng(12)
    K, N, S = 512, 64, 130
    Bs = [rng.integers(-8, 8, size=(K, N), dtype=np.int8) for _ in range(S)]
    ws = [ctx.i4_pack(B) for B in Bs]
    As = [rng.integers(-8, 8, size=(1 + i % 4, K), dtype=np.int8) for i in range(S)]
    Cs = [np.zeros((A.shape[0], N), np.int32) for A in As]
    arr = (TaskI4 * S)(*[TaskI4(w.h, A.shape[0], A.ctypes.data, Cm.ctypes.data) for w, A, Cm in zip(ws, As, Cs)])
    l0 = ctx.launches()
    assert ctx.L.ork_i4_mm_run_experts(ctx.ctx, arr, S, 3) == 0
    assert ctx.launches() - l0 == 2  # 96 + 34 tasks
    for B, A, Cm in zip(Bs, As, Cs):
        assert np.array_equal(Cm, of.gemm_i32(A, B))
    assert ctx.L.ork_i4_mm_run_chain(ctx.ctx, S, arr) == 0
    for w in ws:
        w.free()


def test_chain_async_device_pointers_and_stream_alias(ctx):
    import torch

    L = ork_b200.lib()
    rng = np.random.default_rng(13)
    dev = torch.device("cuda", L.ork_b200_device(ctx.ctx))
    shapes = [(1024, 128), (2048, 64), (512, 256)]
    Bs = [rng.integers(-128, 128, size=s, dtype=np.int8) for s in shapes]
    ws = [ctx.i8_pack(B) for B in Bs]
    As = [rng.integers(-128, 128, size=(4, s[0]), dtype=np.int8) for s in shapes]
    tA = [torch.from_numpy(A).to(dev) for A in As]
    tC = [torch.zeros((4, s[1] + 8), dtype=torch.int32, device=dev) for s in shapes]
    arr = (TaskI8 * 3)(*[TaskI8(w.h, 4, a.data_ptr(), c.data_ptr(), s[1] + 8) for w, a, c, s in zip(ws, tA, tC, shapes)])
    torch.cuda.synchronize()
    assert L.ork_b200_i8_mm_run_chain_async(ctx.ctx, 3, arr) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    for B, A, c, s in zip(Bs, As, tC, shapes):
        got = c.cpu().numpy()
        assert np.array_equal(got[:, :s[1]], of.gemm_i32(A, B)) and not got[:, s[1]:].any()
    # the synchronous stream entry point is the same batch
    Ch = [np.zeros((4, s[1]), np.int32) for s in shapes]
    arr2 = (TaskI8 * 3)(*[TaskI8(w.h, 4, A.ctypes.data, Cm.ctypes.data, 0) for w, A, Cm in zip(ws, As, Ch)])
    assert L.ork_i8_mm_run_stream(ctx.ctx, 3, arr2) == 0
    for B, A, Cm in zip(Bs, As, Ch):
        assert np.array_equal(Cm, of.gemm_i32(A, B))
    for w in ws:
        w.free()


def test_chain_refusals(ctx):
    L = ctx.L
    K, N = 256, 64
    w8 = ctx.i8_pack(np.ones((K, N), np.int8))
    w4 = ctx.i4_pack(np.ones((K, N), np.int8))
    wf = ctx.f16_pack(np.ones((K, N), np.float16))
    A = np.ones((2, K), np.int8)
    Cm = np.zeros((2, N), np.int32)

    def one(w, M=2, a=A, c=Cm, cs=0):
        return (TaskI8 * 1)(TaskI8(w, M, a.ctypes.data if a is not None else None,
                                   c.ctypes.data if c is not None else None, cs))

    assert L.ork_i8_mm_run_chain(ctx.ctx, 0, None) == 0
    assert L.ork_i8_mm_run_chain(ctx.ctx, 1, None) == -1
    assert L.ork_i8_mm_run_chain(None, 1, one(w8.h)) == -1
    assert L.ork_i8_mm_run_chain(ctx.ctx, 1, one(None)) == -1
    assert L.ork_i8_mm_run_chain(ctx.ctx, 1, one(w4.h)) == -1    # W4A4 weight in an int8 batch
    assert L.ork_i8_mm_run_chain(ctx.ctx, 1, one(wf.h)) == -1    # fp16 weight
    assert L.ork_i8_mm_run_chain(ctx.ctx, 1, one(w8.h, M=0)) == -1
    assert L.ork_i8_mm_run_chain(ctx.ctx, 1, one(w8.h, a=None)) == -1
    assert L.ork_i8_mm_run_chain(ctx.ctx, 1, one(w8.h, cs=N - 16)) == -1
    shared = np.zeros(4096, np.int8)
    t = (TaskI8 * 1)(TaskI8(w8.h, 2, shared.ctypes.data, shared.ctypes.data + 128, 0))
    assert L.ork_i8_mm_run_chain(ctx.ctx, 1, t) == -1           # A/C overlap
    t4 = (TaskI4 * 1)(TaskI4(w8.h, 2, A.ctypes.data, Cm.ctypes.data))
    assert L.ork_i4_mm_run_chain(ctx.ctx, 1, t4) == -1          # int8 weight in a W4A4 batch
    assert L.ork_i8_mm_run_chain(ctx.ctx, 1, one(w8.h)) == 0 and np.all(Cm == K)
    for w in (w8, w4, wf):
        w.free()


def test_submit_collect_ring(ctx):
    L = ctx.L
    rng = np.random.default_rng(14)
    K, N = 1024, 128
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    Bh = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    w8, wh = ctx.i8_pack(B), ctx.f16_pack(Bh)
    As = [rng.integers(-128, 128, size=(1 + i, K), dtype=np.int8) for i in range(7)]
    Ah = rng.uniform(-1, 1, size=(3, K)).astype(np.float16)
    tickets = [L.ork_mm_submit(ctx.ctx, w8.h, A.shape[0], _p(A)) for A in As]
    th = L.ork_mm_submit(ctx.ctx, wh.h, 3, _p(Ah))
    assert all(t >= 0 for t in tickets) and th >= 0
    assert L.ork_mm_submit(ctx.ctx, w8.h, 1, _p(As[0])) == -1  # all 8 slots in flight
    Cf = np.zeros((3, N), np.float32)
    assert L.ork_mm_collect(ctx.ctx, th, _p(Cf)) == 0
    assert np.abs(Cf - of.gemm_f16(Ah, Bh)).max() <= 1e-3 * np.sqrt(K) * np.abs(Ah).max() * np.abs(Bh).max()
    for t, A in reversed(list(zip(tickets, As))):  # out of order
        Cm = np.zeros((A.shape[0], N), np.int32)
        assert L.ork_mm_collect(ctx.ctx, t, _p(Cm)) == 0
        assert np.array_equal(Cm, of.gemm_i32(A, B))
    Cm = np.zeros((1, N), np.int32)
    assert L.ork_mm_collect(ctx.ctx, tickets[0], _p(Cm)) == -1  # already collected
    assert L.ork_mm_collect(ctx.ctx, 12345, _p(Cm)) == -1
    t = L.ork_mm_submit(ctx.ctx, w8.h, 1, _p(As[0]))  # slots are reusable
    assert t >= 0 and L.ork_mm_collect(ctx.ctx, t, _p(Cm)) == 0 and np.array_equal(Cm, of.gemm_i32(As[0], B))
    w8.free()
    wh.free()
