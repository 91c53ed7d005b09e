"""The glue around int8 matmuls on the B200 (include/ork_b200.h: ork_b200_rmsnorm_q8_async,
ork_b200_argmax_scaled_async, and the row forms ork_b200_rows_q8_async / _rows_swiglu_q8_async /
_rows_dequant_async / _rows_qk_rope_async): RMSNorm + per-tensor int8 quantization and SwiGLU + quantization against the oracle's restatement of the
reference's CPU glue (src/spine_kernels.h spine_rmsnorm + spine_quant; the sum of squares is reduced in a
different order on the GPU, so a code may differ by one at a rounding boundary and the scale by an ulp),
and the greedy pick against numpy's first-maximum argmax, including ties, repeated calls (the scratch is
cleared for the next call) and CUDA-graph replay. Refusals as documented."""
import ctypes as C

import numpy as np
import pytest

import oracle_ffi as of

pytestmark = pytest.mark.gpu


def _dev(ctx):
    import torch

    return torch.device("cuda", ctx.L.ork_b200_device(ctx.ctx))


@pytest.mark.parametrize("n,gain", [(2048, True), (5000, True), (8192, False), (1, True), (37, False)])
def test_rmsnorm_q8_matches_oracle(ctx, n, gain):
    import torch

    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 3.0).astype(np.float32)
    g = (0.5 + rng.random(n)).astype(np.float32) if gain else None
    want_q, want_s = of.rms_q8(x, g)
    dev = _dev(ctx)
    tx = torch.from_numpy(x).to(dev)
    tg = torch.from_numpy(g).to(dev) if gain else None
    q = torch.zeros(n, dtype=torch.int8, device=dev)
    s = torch.zeros(1, dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    assert ctx.L.ork_b200_rmsnorm_q8_async(ctx.ctx, tx.data_ptr(), tg.data_ptr() if gain else None, n, q.data_ptr(),
                                          s.data_ptr()) == 0
    assert ctx.L.ork_b200_sync(ctx.ctx) == 0
    got_q, got_s = q.cpu().numpy(), float(s.item())
    assert abs(got_s - want_s) <= 2e-6 * abs(want_s)
    d = np.abs(got_q.astype(np.int32) - want_q.astype(np.int32))
    assert d.max() <= 1 and (d > 0).mean() <= 0.01, (d.max(), (d > 0).mean())


def test_rmsnorm_q8_refusals(ctx):
    import torch

    dev = _dev(ctx)
    x = torch.ones(9000, device=dev)
    q = torch.zeros(9000, dtype=torch.int8, device=dev)
    L = ctx.L
    assert L.ork_b200_rmsnorm_q8_async(ctx.ctx, x.data_ptr(), None, 0, q.data_ptr(), None) == -1
    assert L.ork_b200_rmsnorm_q8_async(ctx.ctx, x.data_ptr(), None, 8193, q.data_ptr(), None) == -1
    assert L.ork_b200_rmsnorm_q8_async(ctx.ctx, None, None, 16, q.data_ptr(), None) == -1
    assert L.ork_b200_rmsnorm_q8_async(ctx.ctx, x.data_ptr(), None, 16, None, None) == -1
    assert L.ork_b200_rmsnorm_q8_async(ctx.ctx, x.data_ptr(), None, 16, q.data_ptr(), None) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    assert np.all(q[:16].cpu().numpy() == 127)


def _pick(ctx, C_, bs, n):
    import torch

    idx = torch.full((1,), -7, dtype=torch.int64, device=C_.device)
    assert ctx.L.ork_b200_argmax_scaled_async(ctx.ctx, C_.data_ptr(), bs.data_ptr(), n, idx.data_ptr()) == 0
    assert ctx.L.ork_b200_sync(ctx.ctx) == 0
    return int(idx.item())


def test_argmax_scaled(ctx):
    import torch

    dev = _dev(ctx)
    rng = np.random.default_rng(11)
    for n in (151936, 1, 513, 100000):
        c = rng.integers(-(1 << 22), 1 << 22, size=n, dtype=np.int32)
        bs = (rng.random(n) * 0.02 + 1e-4).astype(np.float32)
        want = int(np.argmax(c.astype(np.float32) * bs))
        got = _pick(ctx, torch.from_numpy(c).to(dev), torch.from_numpy(bs).to(dev), n)
        assert got == want, (n, got, want)
    # ties: the first index wins; all-negative rows; twice in a row (the scratch is cleared)
    c = np.full(4096, -5, np.int32)
    c[[100, 7, 3000]] = 9
    bs = np.ones(4096, np.float32)
    for _ in range(2):
        assert _pick(ctx, torch.from_numpy(c).to(dev), torch.from_numpy(bs).to(dev), 4096) == 7
    c = -np.arange(1, 1001, dtype=np.int32)
    assert _pick(ctx, torch.from_numpy(c).to(dev), torch.ones(1000, device=dev), 1000) == 0


def test_argmax_scaled_graph_replay(ctx):
    import torch

    dev = _dev(ctx)
    L = ctx.L
    n = 65536
    Cd = torch.zeros(n, dtype=torch.int32, device=dev)
    bs = torch.ones(n, dtype=torch.float32, device=dev)
    idx = torch.zeros(1, dtype=torch.int64, device=dev)
    s = torch.cuda.ExternalStream(L.ork_b200_stream(ctx.ctx))
    assert L.ork_b200_argmax_scaled_async(ctx.ctx, Cd.data_ptr(), bs.data_ptr(), n, idx.data_ptr()) == 0
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        assert L.ork_b200_argmax_scaled_async(ctx.ctx, Cd.data_ptr(), bs.data_ptr(), n, idx.data_ptr()) == 0
    for j in (12345, 77, n - 1):
        Cd.zero_()
        Cd[j] = 1
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        assert int(idx.item()) == j
    del graph


def test_argmax_scaled_refusals(ctx):
    L = ctx.L
    buf = (C.c_int32 * 4)()
    assert L.ork_b200_argmax_scaled_async(ctx.ctx, None, None, 4, None) == -1
    assert L.ork_b200_argmax_scaled_async(None, C.addressof(buf), C.addressof(buf), 4, C.addressof(buf)) == -1
    assert L.ork_b200_argmax_scaled_async(ctx.ctx, C.addressof(buf), C.addressof(buf), 0, C.addressof(buf)) == -1


def test_rows_q8_norm_and_plain(ctx):
    import torch

    dev = _dev(ctx)
    rng = np.random.default_rng(21)
    rows, n = 128, 2048
    x = (rng.standard_normal((rows, n)) * 2.0).astype(np.float32)
    g = (0.5 + rng.random(n)).astype(np.float32)
    tx, tg = torch.from_numpy(x).to(dev), torch.from_numpy(g).to(dev)
    q = torch.zeros((rows, n), dtype=torch.int8, device=dev)
    s = torch.zeros(rows, dtype=torch.float32, device=dev)
    L = ctx.L
    # RMSNorm + quantization against the oracle, row by row
    assert L.ork_b200_rows_q8_async(ctx.ctx, tx.data_ptr(), tg.data_ptr(), rows, n, 1, q.data_ptr(), s.data_ptr()) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    gq, gs = q.cpu().numpy(), s.cpu().numpy()
    for m in range(0, rows, 17):
        wq, ws = of.rms_q8(x[m], g)
        assert abs(gs[m] - ws) <= 2e-6 * ws
        assert np.abs(gq[m].astype(int) - wq.astype(int)).max() <= 1
    # plain quantization: no reduction order involved, so exact
    assert L.ork_b200_rows_q8_async(ctx.ctx, tx.data_ptr(), None, rows, n, 0, q.data_ptr(), s.data_ptr()) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    f = np.float32
    ws = (f(127.0) / np.maximum(f(1e-6), np.abs(x).max(axis=1))).astype(f)
    wq = np.clip(np.rint((x * ws[:, None]).astype(f)), -127, 127).astype(np.int8)
    assert np.array_equal(s.cpu().numpy(), ws) and np.array_equal(q.cpu().numpy(), wq)


def test_rows_swiglu_q8_and_dequant(ctx):
    import torch

    dev = _dev(ctx)
    rng = np.random.default_rng(22)
    rows, n = 64, 6144
    cg = rng.integers(-60000, 60000, size=(rows, n)).astype(np.int32)
    cu = rng.integers(-60000, 60000, size=(rows, n)).astype(np.int32)
    sin = (5000.0 + 5000.0 * rng.random(rows)).astype(np.float32)
    tg, tu, ts = (torch.from_numpy(a).to(dev) for a in (cg, cu, sin))
    q = torch.zeros((rows, n), dtype=torch.int8, device=dev)
    s = torch.zeros(rows, dtype=torch.float32, device=dev)
    L = ctx.L
    assert L.ork_b200_rows_swiglu_q8_async(ctx.ctx, tg.data_ptr(), tu.data_ptr(), rows, n, ts.data_ptr(), q.data_ptr(),
                                          s.data_ptr()) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    gq, gs = q.cpu().numpy(), s.cpu().numpy()
    for m in range(0, rows, 9):
        wq, ws = of.swiglu_q8(cg[m], cu[m], sin[m])
        assert abs(gs[m] - ws) <= 1e-6 * ws
        assert np.abs(gq[m].astype(int) - wq.astype(int)).max() <= 1
    # dequantization with per-channel scales and a residual: one IEEE op at a time, so exact
    f = np.float32
    bs = (rng.random(n) * 0.01).astype(f)
    res = rng.standard_normal((rows, n)).astype(f)
    tb, tr = torch.from_numpy(bs).to(dev), torch.from_numpy(res).to(dev)
    out = torch.zeros((rows, n), dtype=torch.float32, device=dev)
    assert L.ork_b200_rows_dequant_async(ctx.ctx, tg.data_ptr(), rows, n, ts.data_ptr(), tb.data_ptr(), tr.data_ptr(),
                                        out.data_ptr()) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    want = (res + ((cg.astype(f) / sin[:, None]).astype(f) * bs).astype(f)).astype(f)
    assert np.array_equal(out.cpu().numpy(), want)
    plain = torch.zeros((rows, n), dtype=torch.float32, device=dev)
    assert L.ork_b200_rows_dequant_async(ctx.ctx, tu.data_ptr(), rows, n, ts.data_ptr(), None, None,
                                        plain.data_ptr()) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    assert np.array_equal(plain.cpu().numpy(), (cu.astype(f) / sin[:, None]).astype(f))
    assert L.ork_b200_rows_q8_async(ctx.ctx, tr.data_ptr(), None, rows, 8193, 0, q.data_ptr(), None) == -1
    assert L.ork_b200_rows_dequant_async(ctx.ctx, tg.data_ptr(), 0, n, ts.data_ptr(), None, None, out.data_ptr()) == -1


@pytest.mark.parametrize("dk,gains", [(128, True), (64, False), (256, True)])
def test_rows_qk_rope(ctx, dk, gains):
    """q / k head RMSNorm + RoPE NeoX over rows at positions pos0 + t (the decode layer's head_vec), q
    written head-major, k and v into the caches at those rows, other cache rows untouched; against a
    float64 restatement (float32 angles of a few hundred radians are off by ~2e-5 rad: tolerance 2e-4 of
    the head's magnitude)."""
    import torch

    dev = _dev(ctx)
    rng = np.random.default_rng(dk)
    T, H, Hkv, pos0, hstride, base = 37, 4, 2, 300, 400, 1e6
    q = rng.standard_normal((T, H * dk)).astype(np.float32)
    k = rng.standard_normal((T, Hkv * dk)).astype(np.float32)
    v = rng.standard_normal((T, Hkv * dk)).astype(np.float32)
    qg = (0.5 + rng.random(dk)).astype(np.float32) if gains else None
    kg = (0.5 + rng.random(dk)).astype(np.float32) if gains else None
    tq, tk, tv = (torch.from_numpy(a).to(dev) for a in (q, k, v))
    tqg = torch.from_numpy(qg).to(dev) if gains else None
    tkg = torch.from_numpy(kg).to(dev) if gains else None
    qo = torch.zeros((H, T, dk), device=dev)
    Kc = torch.full((Hkv, hstride, dk), 7.0, device=dev)
    Vc = torch.full((Hkv, hstride, dk), 7.0, device=dev)
    L = ctx.L
    assert L.ork_b200_rows_qk_rope_async(ctx.ctx, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), T, H, Hkv, dk,
                                         tqg.data_ptr() if gains else None, tkg.data_ptr() if gains else None, pos0,
                                         base, qo.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), hstride) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0

    def head(x, g, pos):
        x = x.astype(np.float64)
        if g is not None:
            x = x / np.sqrt((x * x).sum() / dk + 1e-6) * g
        th = pos * np.power(base, -2.0 * np.arange(dk // 2) / dk)
        a, b = x[: dk // 2].copy(), x[dk // 2:].copy()
        return np.concatenate([a * np.cos(th) - b * np.sin(th), a * np.sin(th) + b * np.cos(th)])

    gq, gK, gV = qo.cpu().numpy(), Kc.cpu().numpy(), Vc.cpu().numpy()
    for t in range(0, T, 6):
        for h in range(H):
            w = head(q[t, h * dk:(h + 1) * dk], qg, pos0 + t)
            assert np.abs(gq[h, t] - w).max() <= 2e-4 * np.abs(w).max(), (t, h)
        for h in range(Hkv):
            w = head(k[t, h * dk:(h + 1) * dk], kg, pos0 + t)
            assert np.abs(gK[h, pos0 + t] - w).max() <= 2e-4 * np.abs(w).max(), (t, h)
            assert np.array_equal(gV[h, pos0 + t], v[t, h * dk:(h + 1) * dk])
    assert np.all(gK[:, :pos0] == 7.0) and np.all(gK[:, pos0 + T:] == 7.0)
    assert L.ork_b200_rows_qk_rope_async(ctx.ctx, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), T, H, Hkv, 96, None,
                                         None, 0, base, qo.data_ptr(), Kc.data_ptr(), Vc.data_ptr(), hstride) == -1
    assert L.ork_b200_rows_qk_rope_async(ctx.ctx, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), T, H, Hkv, dk, None,
                                         None, hstride - T + 1, base, qo.data_ptr(), Kc.data_ptr(), Vc.data_ptr(),
                                         hstride) == -1
