"""The restated decode layer against ork-driver's own glue kernels (host, no GPU).

ork_i8_mm_layer's direct path (src/npu/i8/chain.c:106-122) lives in a translation unit that only builds
for aarch64; oracle/ref_layer.c drives the reference's own glue kernels (src/spine_kernels.h) and exact
int32 GEMM in the same order, compiled from the reference sources. The restatement (oracle/ork_oracle.c
orc_layer_i8) must reproduce it bit for bit.
"""
import numpy as np
import pytest

import oracle_ffi as of


@pytest.mark.parametrize("dims", [
    dict(D=256, H=4, Hkv=2, dk=64, dv=64, Nff=512, nkv=17, pos=17),
    dict(D=512, H=8, Hkv=8, dk=64, dv=64, Nff=1024, nkv=1, pos=0),
    dict(D=2048, H=16, Hkv=8, dk=128, dv=128, Nff=6144, nkv=100, pos=100),
])
def test_restated_layer_equals_reference_glue(dims):
    ref = of.reference()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    Bs, norms, x, Kc, Vc = of.layer_inputs(7, dims["D"], dims["H"], dims["Hkv"], dims["dk"], dims["Nff"],
                                           dims["nkv"], dims["pos"])
    scale, base = 1.0 / np.sqrt(dims["dk"]), 1e6
    got, _, _ = of.layer(dims, scale, base, Bs, norms, x, Kc, Vc)
    dm = np.array([dims[k] for k in of.LAYER_KEYS], np.uint32)
    want = np.zeros(dims["D"], np.float32)
    assert ref.ref_layer_i8(of._p(dm), scale, base, *[of._p(np.ascontiguousarray(b)) for b in Bs],
                            of._p(norms[0]), of._p(norms[1]), of._p(norms[2]), of._p(x), of._p(Kc), of._p(Vc),
                            of._p(want)) == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.isfinite(got).all() and np.abs(got - x).max() > 0


def test_kv_extension_appends_then_attends():
    """With the extension the caches gain the token's k/v at slot nkv; without it they are read only."""
    dims = dict(D=256, H=4, Hkv=2, dk=64, dv=64, Nff=512, nkv=5, pos=5)
    Bs, norms, x, Kc, Vc = of.layer_inputs(8, 256, 4, 2, 64, 512, 5, 5, hstride=8)
    out0, K0, V0 = of.layer(dims, 0.125, 1e4, Bs, norms, x, Kc, Vc)
    assert np.array_equal(K0, Kc) and np.array_equal(V0, Vc)
    out1, K1, V1 = of.layer(dims, 0.125, 1e4, Bs, norms, x, Kc, Vc, kv_ext=True, hstride=8)
    assert np.array_equal(K1[:, :5], Kc[:, :5]) and K1[:, 5].any() and V1[:, 5].any()
    assert not K1[:, 6:].any()
    assert not np.array_equal(out0, out1)
