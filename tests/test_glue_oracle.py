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
