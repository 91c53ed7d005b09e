"""The decode layer (ork_i8_mm_layer, ork-driver include/ork/chain.h:105-110) on the B200 against the
restated layer of oracle/ork_oracle.c, itself pinned bit for bit to the reference's own glue kernels
(tests/test_layer_host.py). Every case runs in both of the library's forms: the persistent one-launch
kernel (layer_fused.cu, the default where the seven weights share a format) and the multi-launch form
(layer.cu, ORKB_LAYER_FUSED=0).

The matmuls are exact int32 on both sides; the fp32 glue differs only in summation order (tree vs
sequential) and in CUDA's expf/sinf/cosf/powf against the host's, a few ulps each. Those ulps can move a
value across an int8 rounding boundary in the three intermediate quantizations, which changes that one
code by 1 and the layer output by about |w| / s -- far below 1 % of the output's scale. The bound below
(3e-3 of max|x_out|) admits a few such flips and nothing larger.
"""
import ctypes as C

import numpy as np
import pytest

import oracle_ffi as of
import ork_b200
from ork_b200 import LayerDims, LayerKV, LayerW

pytestmark = pytest.mark.gpu
_p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
TOL = 3e-3

# attention splits each head's keys over CTAs in chunks of at least 32: one chunk, several, and (9000 keys)
# more chunks than a head may have CTAs, so chunks of 64. The 9000-key case rotates at position 100: at
# position 9000 the RoPE angle pos * base^(-2i/dk) is so ill-conditioned that a one-ulp change of the base
# alone moves the oracle's own output by 0.8 % (5e-7 at position 100), so CUDA's powf / cosf against the
# host's would be measured there, not the kernel.
DIMS = [dict(D=256, H=4, Hkv=2, dk=64, dv=64, Nff=512, nkv=17, pos=17),
        dict(D=2048, H=16, Hkv=8, dk=128, dv=128, Nff=6144, nkv=100, pos=100),
        dict(D=512, H=8, Hkv=2, dk=128, dv=128, Nff=1024, nkv=3000, pos=3000),
        dict(D=512, H=8, Hkv=2, dk=128, dv=128, Nff=1024, nkv=9000, pos=100)]


@pytest.fixture(params=["fused", "multi"])
def path(request, tune):
    tune("ORKB_LAYER_FUSED", "1" if request.param == "fused" else "0")
    return request.param


def _pack(ctx, Bs):
    return [ctx.i8_pack(b) for b in Bs]


def _dims(d, scale, base):
    return LayerDims(*[d[k] for k in of.LAYER_KEYS], scale, base)


def _close(got, want):
    err = np.abs(got - want).max()
    return err <= TOL * np.abs(want).max(), err


def _run(ctx, d, ws, norms, x, Kc, Vc, scale, base):
    out = np.zeros(d["D"], np.float32)
    dims = _dims(d, scale, base)
    l0 = ctx.launches()
    rc = ctx.L.ork_i8_mm_layer(ctx.ctx, C.byref(dims), *[w.h for w in ws], _p(norms[0]), _p(norms[1]),
                               _p(norms[2]), _p(x), _p(Kc), _p(Vc), _p(out))
    assert rc == 0
    return out, ctx.launches() - l0


@pytest.mark.parametrize("d", DIMS)
def test_layer_matches_oracle(ctx, path, d):
    Bs, norms, x, Kc, Vc = of.layer_inputs(21, d["D"], d["H"], d["Hkv"], d["dk"], d["Nff"], d["nkv"], d["pos"])
    scale, base = 1.0 / np.sqrt(d["dk"]), 1e6
    want, _, _ = of.layer(d, scale, base, Bs, norms, x, Kc, Vc)
    ws = _pack(ctx, Bs)
    out, launches = _run(ctx, d, ws, norms, x, Kc, Vc, scale, base)
    for w in ws:
        w.free()
    ok, err = _close(out, want)
    print("max|err|", err, "scale", np.abs(want).max())
    assert ok, err
    assert launches == 1 if path == "fused" else launches >= 9


@pytest.mark.parametrize("fmt", ["u4", "nf4", "mixed"])
def test_layer_int4_weights(ctx, env_clean, path, fmt):
    """int4-weight / int8-activation stores (uniform and NF4 codes): the oracle runs the same layer on the
    int8 codes the stores hold. A mix of formats takes the multi-launch form in both settings."""
    d = DIMS[1]
    Bs, norms, x, Kc, Vc = of.layer_inputs(25, d["D"], d["H"], d["Hkv"], d["dk"], d["Nff"], d["nkv"], d["pos"])
    rng = np.random.default_rng(26)
    ws, codes = [], []
    for i, B in enumerate(Bs):
        K, N = B.shape
        if fmt == "mixed" and i % 2:
            ws.append(ctx.i8_pack(B))
            codes.append(B)
            continue
        if fmt == "nf4" or (fmt == "mixed" and i == 2):
            env_clean.setenv("ORK_NF4", "1")
        w, _ = ctx.i4a8_pack(rng.standard_normal((N, K), dtype=np.float32))
        env_clean.delenv("ORK_NF4", raising=False)
        ws.append(w)
        codes.append(of.i4a8_blob_codes(w.dump(), K, N)[0])
    scale, base = 1.0 / np.sqrt(d["dk"]), 1e6
    want, _, _ = of.layer(d, scale, base, codes, norms, x, Kc, Vc)
    out, launches = _run(ctx, d, ws, norms, x, Kc, Vc, scale, base)
    for w in ws:
        w.free()
    ok, err = _close(out, want)
    assert ok, err
    assert launches == 1 if (path == "fused" and fmt != "mixed") else launches >= 9


@pytest.mark.parametrize("p0,cap", [(5, 16), (95, 160)])
def test_layer_decode_extension_graph_replay(ctx, path, p0, cap):
    """Three decode steps captured once in a CUDA graph: each step appends its k/v at the device position
    and attends over it, the position advancing on the device; compared step by step with the oracle.
    From position 95 the token's own key sits in the last of several key chunks, and the steps cross a
    chunk boundary (96 keys -> 97)."""
    import torch

    L = ork_b200.lib()
    d = dict(D=256, H=4, Hkv=2, dk=64, dv=64, Nff=512, nkv=p0, pos=p0)
    Bs, norms, x0, Kc, Vc = of.layer_inputs(22, 256, 4, 2, 64, 512, p0, p0, hstride=cap)
    scale, base = 0.125, 1e4
    ws = _pack(ctx, Bs)
    dev = torch.device("cuda", L.ork_b200_device(ctx.ctx))
    t = {k: torch.from_numpy(v).to(dev) for k, v in dict(an=norms[0], qn=norms[1], fn=norms[2], kn=norms[3],
                                                         x=x0, K=Kc, V=Vc).items()}
    xo = torch.zeros(256, dtype=torch.float32, device=dev)
    pos = torch.tensor([p0], dtype=torch.int32, device=dev)
    kv = LayerKV(t["kn"].data_ptr(), 1, cap, pos.data_ptr())
    dims = _dims(d, scale, base)
    stream = torch.cuda.ExternalStream(L.ork_b200_stream(ctx.ctx))

    def step():
        assert L.ork_b200_i8_mm_layer_async(ctx.ctx, C.byref(dims), *[w.h for w in ws], t["an"].data_ptr(),
                                       t["qn"].data_ptr(), t["fn"].data_ptr(), t["x"].data_ptr(),
                                       t["K"].data_ptr(), t["V"].data_ptr(), xo.data_ptr(), C.byref(kv)) == 0
        t["x"].copy_(xo)  # the next step's input is this step's output
        pos.add_(1)

    # one eager call sizes the layer workspace before capture (its result is discarded: a scratch cache)
    sK, sV, sp = t["K"].clone(), t["V"].clone(), pos.clone()
    kv0 = LayerKV(t["kn"].data_ptr(), 1, cap, sp.data_ptr())
    assert L.ork_b200_i8_mm_layer_async(ctx.ctx, C.byref(dims), *[w.h for w in ws], t["an"].data_ptr(),
                                   t["qn"].data_ptr(), t["fn"].data_ptr(), t["x"].data_ptr(), sK.data_ptr(),
                                   sV.data_ptr(), xo.data_ptr(), C.byref(kv0)) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        step()
    # the capture ran nothing: replay three steps from position p0
    refK, refV, x = Kc.copy(), Vc.copy(), x0.copy()
    for s in range(3):
        g.replay()
        torch.cuda.synchronize()
        ds = dict(d, nkv=p0 + s, pos=p0 + s)
        want, refK, refV = of.layer(ds, scale, base, Bs, norms, x, refK, refV, kv_ext=True, hstride=cap)
        got = xo.cpu().numpy()
        ok, err = _close(got, want)
        assert ok, (s, err)
        gotK = t["K"].cpu().numpy()
        assert np.abs(gotK[:, p0 + s] - refK[:, p0 + s]).max() <= 1e-3 * np.abs(refK[:, p0 + s]).max(), s
        x = want
    assert int(pos.item()) == p0 + 3
    for w in ws:
        w.free()


def test_layer_device_position_past_capacity_is_an_error(ctx, path):
    """A device-read position whose token would not fit the caches: the kernel's own check skips attention
    (no cache access), the sync reports the error once, and the context keeps working."""
    import torch

    L = ork_b200.lib()
    cap = 8
    d = dict(D=256, H=4, Hkv=2, dk=64, dv=64, Nff=512, nkv=cap, pos=cap)
    Bs, norms, x0, Kc, Vc = of.layer_inputs(24, 256, 4, 2, 64, 512, 4, 4, hstride=cap)
    ws = _pack(ctx, Bs)
    dev = torch.device("cuda", L.ork_b200_device(ctx.ctx))
    t = {k: torch.from_numpy(v).to(dev) for k, v in dict(an=norms[0], qn=norms[1], fn=norms[2], kn=norms[3],
                                                         x=x0, K=Kc, V=Vc).items()}
    K0 = t["K"].clone()
    xo = torch.zeros(256, dtype=torch.float32, device=dev)
    dims = _dims(d, 0.125, 1e4)

    def call(p):
        pos = torch.tensor([p], dtype=torch.int32, device=dev)
        kv = LayerKV(t["kn"].data_ptr(), 1, cap, pos.data_ptr())
        torch.cuda.synchronize()
        assert L.ork_b200_i8_mm_layer_async(ctx.ctx, C.byref(dims), *[w.h for w in ws], t["an"].data_ptr(),
                                       t["qn"].data_ptr(), t["fn"].data_ptr(), t["x"].data_ptr(),
                                       t["K"].data_ptr(), t["V"].data_ptr(), xo.data_ptr(), C.byref(kv)) == 0
        return L.ork_b200_sync(ctx.ctx)

    assert call(cap) == -1                      # slot cap is past the caches
    assert torch.equal(t["K"], K0)              # nothing was written
    assert call(cap - 1) == 0                   # the last slot is fine, and the flag was cleared
    assert not torch.equal(t["K"], K0)
    for w in ws:
        w.free()


def test_layer_refusals(ctx, path):
    d = DIMS[0]
    Bs, norms, x, Kc, Vc = of.layer_inputs(23, d["D"], d["H"], d["Hkv"], d["dk"], d["Nff"], d["nkv"], d["pos"])
    ws = _pack(ctx, Bs)
    out = np.zeros(d["D"], np.float32)
    L = ctx.L

    def call(dd, wl=None, xx=x):
        dims = _dims(dd, 0.125, 1e4)
        wl = wl or ws
        return L.ork_i8_mm_layer(ctx.ctx, C.byref(dims), *[w.h if w else None for w in wl], _p(norms[0]),
                                 _p(norms[1]), _p(norms[2]), None if xx is None else _p(xx), _p(Kc), _p(Vc), _p(out))

    assert call(dict(d, dv=32)) == -3          # dv != dk
    assert call(dict(d, Hkv=3)) == -3          # H % Hkv
    assert call(dict(d, nkv=0)) == -3          # nothing to attend to
    assert call(d, wl=[ws[1]] + ws[1:]) == -3  # q weight of the wrong shape
    assert call(d, xx=None) == -3
    wf = ctx.f16_pack(np.zeros((d["D"], 256), np.float16))
    assert call(d, wl=[wf] + ws[1:]) == -3     # not an int8-compute weight
    wf.free()
    assert call(d) == 0
    for w in ws:
        w.free()


@pytest.mark.parametrize("p0,cap", [(5, 16), (70, 96)])
def test_layers_stack_graph_replay(ctx, path, p0, cap):
    """ork_b200_i8_mm_layers_async: three layers with their own weights and caches in one call (one persistent
    launch, or nine launches per layer), the token's k/v appended at the device position, captured once
    and replayed for two tokens; each token compared with the oracle layers applied in turn."""
    import torch

    L = ork_b200.lib()
    D, H, Hkv, dk, F, NL = 256, 4, 2, 64, 512, 3
    d = dict(D=D, H=H, Hkv=Hkv, dk=dk, dv=dk, Nff=F, nkv=p0, pos=p0)
    scale, base = 0.125, 1e4
    dev = torch.device("cuda", L.ork_b200_device(ctx.ctx))
    layers, ws, keep = [], [], []
    for l in range(NL):
        Bs, norms, x0, Kc, Vc = of.layer_inputs(60 + l, D, H, Hkv, dk, F, p0, p0, hstride=cap)
        wl = _pack(ctx, Bs)
        t = {k: torch.from_numpy(v).to(dev) for k, v in dict(an=norms[0], qn=norms[1], fn=norms[2], kn=norms[3],
                                                             K=Kc, V=Vc).items()}
        layers.append((Bs, norms, Kc.copy(), Vc.copy()))
        ws.append(wl)
        keep.append(t)
    x = torch.from_numpy(of.layer_inputs(99, D, H, Hkv, dk, F, 1, 1)[2]).to(dev)
    xo = torch.zeros(D, dtype=torch.float32, device=dev)
    arr = (LayerW * NL)(*[LayerW(*[w.h for w in ws[l]], keep[l]["an"].data_ptr(), keep[l]["qn"].data_ptr(),
                                 keep[l]["fn"].data_ptr(), keep[l]["kn"].data_ptr(), keep[l]["K"].data_ptr(),
                                 keep[l]["V"].data_ptr()) for l in range(NL)])
    dims = _dims(d, scale, base)
    stream = torch.cuda.ExternalStream(L.ork_b200_stream(ctx.ctx))
    # one eager call with the same list of layers before capture (sizes the workspace, uploads the layer
    # table); append off, so the caches are only read
    sp = torch.tensor([p0], dtype=torch.int32, device=dev)
    kv0 = LayerKV(None, 0, cap, sp.data_ptr())
    assert L.ork_b200_i8_mm_layers_async(ctx.ctx, C.byref(dims), NL, arr, x.data_ptr(), xo.data_ptr(), C.byref(kv0)) == 0
    assert L.ork_b200_sync(ctx.ctx) == 0
    pos = torch.tensor([p0], dtype=torch.int32, device=dev)
    kv = LayerKV(None, 1, cap, pos.data_ptr())
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        assert L.ork_b200_i8_mm_layers_async(ctx.ctx, C.byref(dims), NL, arr, x.data_ptr(), xo.data_ptr(),
                                        C.byref(kv)) == 0
        x.copy_(xo)
        pos.add_(1)
    xr = x.cpu().numpy().copy()
    for s in range(2):
        g.replay()
        torch.cuda.synchronize()
        ds = dict(d, nkv=p0 + s, pos=p0 + s)
        for l in range(NL):
            Bs, norms, Kc, Vc = layers[l]
            xr, Kc, Vc = of.layer(ds, scale, base, Bs, norms, xr, Kc, Vc, kv_ext=True, hstride=cap)
            layers[l] = (Bs, norms, Kc, Vc)
        ok, err = _close(xo.cpu().numpy(), xr)
        assert ok, (s, err)
    assert L.ork_b200_sync(ctx.ctx) == 0
    del g
    for wl in ws:
        for w in wl:
            w.free()
