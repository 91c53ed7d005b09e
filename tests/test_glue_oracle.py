"""The oracle's decode glue in front of the LM head (oracle/ork_oracle.c orc_rms_q8: RMSNorm + per-tensor
int8 quantization, the reference's src/spine_kernels.h spine_rmsnorm + spine_quant) against an independent
float32 restatement with the same operation order (sequential sum of squares, x * r * g, 127 / max(1e-6,
max|y|), round half to even, clamp +-127), on CPU."""
import numpy as np

import oracle_ffi as of


def _restated(x, g):
    f = np.float32
    ss = f(0.0)
    for v in x:
        ss = f(ss + f(v * v))
    r = f(f(1.0) / np.sqrt(f(ss / f(x.size)) + f(1e-6), dtype=np.float32))
    y = (x * r).astype(np.float32) * (g if g is not None else f(1.0))
    mx = max(f(1e-6), f(np.abs(y).max()))
    s = f(f(127.0) / mx)
    q = np.clip(np.rint((y * s).astype(np.float32)), -127, 127).astype(np.int8)
    return q, s


def test_rms_q8_against_restatement():
    rng = np.random.default_rng(5)
    for n, gain in ((300, True), (64, False), (1, True)):
        x = (rng.standard_normal(n) * 2.0).astype(np.float32)
        g = (0.5 + rng.random(n)).astype(np.float32) if gain else None
        q, s = of.rms_q8(x, g)
        wq, ws = _restated(x, g)
        assert np.float32(s) == ws
        assert np.array_equal(q, wq)
    q1, _ = of.rms_q8(x, None)
    q2, _ = of.rms_q8(x, np.ones(x.size, np.float32))
    assert np.array_equal(q1, q2)


def test_swiglu_q8_against_restatement():
    rng = np.random.default_rng(9)
    f = np.float32
    cg = rng.integers(-50000, 50000, size=700).astype(np.int32)
    cu = rng.integers(-50000, 50000, size=700).astype(np.int32)
    s = f(9000.0)
    q, sh = of.swiglu_q8(cg, cu, s)
    g = (cg.astype(f) / s).astype(f)
    u = (cu.astype(f) / s).astype(f)
    h = ((g / (f(1.0) + np.exp(-g).astype(f))).astype(f) * u).astype(f)
    mx = max(f(1e-6), f(np.abs(h).max()))
    ws = f(f(127.0) / mx)
    assert abs(f(sh) - ws) <= 1e-6 * ws  # expf of two libms may differ in the last place
    wq = np.clip(np.rint((h * ws).astype(f)), -127, 127).astype(np.int8)
    assert np.abs(q.astype(int) - wq.astype(int)).max() <= 1
