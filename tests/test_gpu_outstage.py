"""Fused output stages on the B200 (ork_i8_mm_run_out8 / _out16 / _ewmul and their _async forms,
ork_i8_npu_ewmul, include/ork/run.h:48-108 and include/ork/sdp.h:45-52), bit-exact against the oracle's
restatement of the reference's requant model (examples/test_mm_i8_out8.c:24-33), over int8 packs and
int4 stores, decode (requant inside the matmul kernel) and prefill (int32 scratch + elementwise pass)
sizes, the gains the reference's own test uses, and its refusals.
"""
import ctypes as C

import numpy as np
import pytest

import oracle_ffi as of
import ork_b200

pytestmark = pytest.mark.gpu
_p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
GAINS = [(0x4000, 14), (0x2000, 14), (0x1000, 15), (0x2AB0, 15), (0x7FFF, 22)]  # test_mm_i8_out8.c:72-80 + one


def _weight(ctx, env, kind, K, N, rng):
    if kind == "i8":
        B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
        return ctx.i8_pack(B), B
    if kind == "nf4":
        env.setenv("ORK_NF4", "1")
    w, _ = ctx.i4a8_pack(rng.standard_normal((N, K), dtype=np.float32))
    env.delenv("ORK_NF4", raising=False)
    return w, of.i4a8_blob_codes(w.dump(), K, N)[0]


@pytest.mark.parametrize("kind", ["i8", "u4", "nf4"])
@pytest.mark.parametrize("M,K,N", [(1, 2048, 2048), (3, 512, 64), (8, 4096, 128), (17, 1024, 256),
                                   (130, 2048, 192)])
def test_stages_match_oracle(ctx, env_clean, kind, M, K, N):
    rng = np.random.default_rng(M * 7 + K + N)
    w, B = _weight(ctx, env_clean, kind, K, N, rng)
    A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
    G = rng.integers(-128, 128, size=(M, N), dtype=np.int8)
    acc = of.gemm_i32(A, B)
    L = ctx.L
    for mult, shift in GAINS:
        c8 = np.zeros((M, N), np.int8)
        c16 = np.zeros((M, N), np.int16)
        ce = np.zeros((M, N), np.int8)
        assert L.ork_i8_mm_run_out8(ctx.ctx, w.h, M, _p(A), _p(c8), mult, shift) == 0
        assert L.ork_i8_mm_run_out16(ctx.ctx, w.h, M, _p(A), _p(c16), mult, shift) == 0
        assert L.ork_i8_mm_run_ewmul(ctx.ctx, w.h, M, _p(A), _p(G), _p(ce), mult, shift) == 0
        assert np.array_equal(c8, of.requant(acc, mult, shift)), (mult, shift)
        assert np.array_equal(c16, of.requant(acc, mult, shift, 16)), (mult, shift)
        assert np.array_equal(ce, of.requant(acc, mult, shift, 8, G)), (mult, shift)
    w.free()


def test_async_device_pointers_one_launch_at_decode(ctx):
    import torch

    L = ork_b200.lib()
    dev = torch.device("cuda", L.ork_b200_device(ctx.ctx))
    rng = np.random.default_rng(31)
    K, N = 2048, 512
    B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
    w = ctx.i8_pack(B)
    for M in (4, 96):
        A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
        G = rng.integers(-128, 128, size=(M, N), dtype=np.int8)
        tA, tG = torch.from_numpy(A).to(dev), torch.from_numpy(G).to(dev)
        t8 = torch.zeros((M, N), dtype=torch.int8, device=dev)
        t16 = torch.zeros((M, N), dtype=torch.int16, device=dev)
        te = torch.zeros((M, N), dtype=torch.int8, device=dev)
        torch.cuda.synchronize()
        l0 = ctx.launches()
        assert L.ork_b200_i8_mm_run_out8_async(ctx.ctx, w.h, M, tA.data_ptr(), t8.data_ptr(), 0x1000, 15) == 0
        if M <= 8:  # the requant runs in the matmul kernel's store
            assert ctx.launches() - l0 == 1
        assert L.ork_b200_i8_mm_run_out16_async(ctx.ctx, w.h, M, tA.data_ptr(), t16.data_ptr(), 0x1000, 15) == 0
        assert L.ork_b200_i8_mm_run_ewmul_async(ctx.ctx, w.h, M, tA.data_ptr(), tG.data_ptr(), te.data_ptr(), 0x2AB0,
                                           15) == 0
        assert L.ork_b200_sync(ctx.ctx) == 0
        acc = of.gemm_i32(A, B)
        assert np.array_equal(t8.cpu().numpy(), of.requant(acc, 0x1000, 15))
        assert np.array_equal(t16.cpu().numpy(), of.requant(acc, 0x1000, 15, 16))
        assert np.array_equal(te.cpu().numpy(), of.requant(acc, 0x2AB0, 15, 8, G))
    w.free()


@pytest.mark.parametrize("M,N", [(8, 64), (1, 16), (37, 8192), (8176, 32)])
def test_npu_ewmul(ctx, M, N):
    rng = np.random.default_rng(M + N)
    up = rng.integers(-128, 128, size=(M, N), dtype=np.int8)
    si = rng.integers(-128, 128, size=(M, N), dtype=np.int8)
    for mult, shift in [(0x4000, 14), (0x2AB0, 15), (1, 0), (0x7FFF, 31)]:
        out = np.zeros((M, N), np.int8)
        us = C.c_double(-1.0)
        assert ctx.L.ork_i8_npu_ewmul(ctx.ctx, _p(up), _p(si), M, N, mult, shift, _p(out), C.byref(us)) == 0
        want = of.requant(up.astype(np.int32) * si.astype(np.int32), mult, shift)
        assert np.array_equal(out, want), (mult, shift)
        assert us.value >= 0.0


def test_refusals(ctx):
    L = ctx.L
    rng = np.random.default_rng(5)
    A = np.ones((2, 8192), np.int8)    # large enough for every K below
    C8 = np.zeros((2, 64), np.int8)

    def out8(w, M=2, mult=0x4000, shift=14, a=A, c=C8):
        return L.ork_i8_mm_run_out8(ctx.ctx, w.h, M, _p(a) if a is not None else None,
                                    _p(c) if c is not None else None, mult, shift)

    w256 = ctx.i8_pack(np.ones((256, 64), np.int8))
    w8k = ctx.i8_pack(np.ones((8192, 64), np.int8))
    wf = ctx.f16_pack(np.ones((512, 64), np.float16))
    w4 = ctx.i4_pack(np.ones((512, 64), np.int8))
    ok = ctx.i8_pack(np.ones((512, 64), np.int8))
    assert out8(w256) == -2      # K % 512 (src/npu/i8/run.c:443)
    assert out8(w8k) == -2       # K > 4096
    assert out8(wf) == -2        # fp16 weight
    assert out8(w4) == -2        # W4A4 weight
    assert out8(ok, shift=-1) == -2
    assert out8(ok, a=None) == -1
    assert out8(ok, M=0) == 0    # nothing to do, as the reference's loops
    assert out8(ok) == 0 and np.all(C8 == 127)  # 512 * 1 * 1 saturates
    G = np.ones((2, 64), np.int8)
    assert L.ork_i8_mm_run_ewmul(ctx.ctx, ok.h, 2, _p(A), None, _p(C8), 0x4000, 14) == -1
    assert L.ork_i8_mm_run_ewmul(ctx.ctx, ok.h, 2, _p(A), _p(G), _p(C8), 0x4000, 14) == 0
    up = rng.integers(-4, 4, size=(8, 64), dtype=np.int8)
    o = np.zeros_like(up)

    def ew(M, N, mult=0x4000, shift=14):
        return L.ork_i8_npu_ewmul(ctx.ctx, _p(up), _p(up), M, N, mult, shift, _p(o), None)

    assert ew(0, 64) == -2 and ew(8177, 16) == -2 and ew(8, 8) == -2 and ew(1, 24) == -2 and ew(1, 8208) == -2
    assert ew(8, 64, mult=0x8000) == -2 and ew(8, 64, mult=-1) == -2 and ew(8, 64, shift=32) == -2
    assert ew(8, 64) == 0 and np.array_equal(o, up.astype(np.int32) ** 2)
    for w in (w256, w8k, wf, w4, ok):
        w.free()
