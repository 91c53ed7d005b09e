"""Pin the oracle before trusting it (CPU only).

1. The restated oracle (oracle/ork_oracle.c) reproduces the 19 golden checksums hard-coded in the
   reference's own tests (examples/quant.c:72-81, examples/test_matmul.c:84-86, :611-612, :639-641).
2. It agrees byte for byte with the reference's compiled CPU code (oracle/_ref, when built here) and with
   the fixtures that code produced (tests/golden/reference_fixtures.json, which travel without the tree).
"""
import ctypes as C
import hashlib
import json
import os

import numpy as np
import pytest

import oracle_ffi as of
import reference_goldens as rg
from make_fixtures import I4A8_CASES, seeded_imatrix, seeded_weights

FIX = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_fixtures.json")))


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _golden_hash(kind, Ms, A, B):
    h = of.FNV_OFFSET
    for m in Ms:
        Cm = of.gemm_f16(A[:m], B) if kind == "f16" else of.gemm_i32(A[:m], B)
        h = of.fnv64(Cm, h)
    return h


@pytest.mark.parametrize("which", ["quant", "f16", "chain", "check_i8"])
def test_restated_oracle_reproduces_reference_goldens(which):
    n = 0
    for name, kind, Ms, K, N, A, B, gold in rg.cases(of.Lcg, which=(which,)):
        assert _golden_hash(kind, Ms, A, B) == gold, name
        n += 1
    assert n == {"quant": 7, "f16": 2, "chain": 7, "check_i8": 3}[which]


def test_fixtures_pin_restated_i4a8_blob(env_clean):
    for i, (name, K, N, nf4, use_im, sr) in enumerate(I4A8_CASES):
        f = FIX["i4a8"][name]
        w = seeded_weights(f["seed"], N, K)
        im = seeded_imatrix(f["seed"], K) if use_im else None
        blob = of.i4a8_blob(w, im, nf4=bool(nf4), sr=bool(sr))
        assert blob.size == f["blob_bytes"], name
        assert _sha(blob) == f["blob_sha256"], name


def test_fixtures_pin_restated_i8_scales():
    for key, f in FIX["chan_scales"].items():
        w = seeded_weights(f["seed"], f["N"], f["K"])
        _, bs = of.i8_quant_f32(w)
        mx = (bs * np.float32(127)).astype(np.float32)  # not used for the pin; bscale is what ships
        assert _sha(bs) == f["bscale_sha256"], key
        # inv = 127/max is recomputed from the same max the restatement used
        absmax = np.maximum(np.abs(w).max(axis=1), np.float32(1e-9)).astype(np.float32)
        inv = (np.float32(127.0) / absmax).astype(np.float32)
        assert _sha(inv) == f["inv_sha256"], key
        del mx


def test_fixtures_pin_w4a4_gemm():
    for key, f in FIX["w4a4"].items():
        rng = np.random.default_rng(f["seed"])
        B = rng.integers(-8, 8, size=(f["K"], f["N"]), dtype=np.int8)
        A = rng.integers(-8, 8, size=(f["M"], f["K"]), dtype=np.int8)
        assert of.fnv64(of.gemm_i32(A, B)) == f["c_fnv64"], key


# ---- direct comparison with the reference's compiled code (this container, or wherever _ref exists) --
needs_ref = pytest.mark.skipif(of.reference() is None, reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("nf4", [0, 1])
@pytest.mark.parametrize("use_im", [False, True])
@pytest.mark.parametrize("sr", [False, True])
def test_restated_i4a8_equals_reference(env_clean, nf4, use_im, sr):
    from make_fixtures import ref_blob

    ref = of.reference()
    K, N = 1024, 96
    w = seeded_weights(31 + nf4 + 2 * use_im + 4 * sr, N, K)
    im = seeded_imatrix(5, K) if use_im else None
    rblob, _ = ref_blob(ref, w, im, nf4, sr)
    assert np.array_equal(of.i4a8_blob(w, im, nf4=bool(nf4), sr=bool(sr)), rblob)


@needs_ref
@pytest.mark.parametrize("nf4", [0, 1])
def test_restated_blob_decode_equals_reference_offline_load(env_clean, nf4):
    from make_fixtures import ref_blob

    ref = of.reference()
    K, N = 512, 64
    w = seeded_weights(77, N, K)
    blob, _ = ref_blob(ref, w, None, nf4, False)
    ctx = ref.ork_npu_init_offline(b"rk3588")
    try:
        rw = ref.ork_i4a8_mm_load(ctx, K, N, of._p(blob), blob.nbytes)
        assert rw
        rcodes = np.ctypeslib.as_array(ref.ork_w_codes(rw), shape=(K, N)).copy()
        rbs = np.ctypeslib.as_array(ref.ork_w_bscale(rw), shape=(N,)).copy()
        rqk = ref.ork_w_quant_kind(rw)
        ref.ork_w_free(rw)
    finally:
        ref.ork_npu_free(ctx)
    codes, bs, qk = of.i4a8_blob_codes(blob, K, N)
    assert np.array_equal(codes, rcodes) and np.array_equal(bs, rbs) and qk == rqk == nf4


@needs_ref
def test_restated_gemm_equals_reference_offline_run():
    ref = of.reference()
    rng = np.random.default_rng(3)
    for M, K, N in ((1, 64, 32), (7, 320, 96), (33, 1024, 256)):
        A = rng.integers(-128, 128, size=(M, K), dtype=np.int8)
        B = rng.integers(-128, 128, size=(K, N), dtype=np.int8)
        Cr = np.zeros((M, N), np.int32)
        ref.ork_i8_mm_run_cpu(M, K, N, of._p(A), of._p(B), of._p(Cr))
        assert np.array_equal(of.gemm_i32(A, B), Cr)
        assert np.array_equal(of.gemm_i32_nk(A, np.ascontiguousarray(B.T)), Cr)


@needs_ref
def test_reference_offline_path_reproduces_quant_c_goldens():
    """The reference's own offline ork_i8_mm_pack + ork_i8_mm_run reproduce its NPU goldens too."""
    ref = of.reference()
    ctx = ref.ork_npu_init_offline(b"rk3588")
    try:
        for name, kind, Ms, K, N, A, B, gold in rg.cases(of.Lcg, which=("quant",), max_macs=1 << 27):
            w = ref.ork_i8_mm_pack(ctx, K, N, of._p(B))
            h = of.FNV_OFFSET
            for m in Ms:
                Cm = np.zeros((m, N), np.int32)
                assert ref.ork_i8_mm_run(ctx, w, m, of._p(A), of._p(Cm)) == 0
                h = of.fnv64(Cm, h)
            ref.ork_w_free(w)
            assert h == gold, name
    finally:
        ref.ork_npu_free(ctx)


@needs_ref
def test_chan_scales_equal_reference():
    ref = of.reference()
    ref.orki_chan_scales_f32.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    w = seeded_weights(9, 128, 512)
    w[3, :] = 0.0  # all-zero channel: max floors at 1e-9
    inv = np.zeros(128, np.float32)
    bs = np.zeros(128, np.float32)
    ref.orki_chan_scales_f32(of._p(w), 512, 128, of._p(inv), of._p(bs))
    _, mine = of.i8_quant_f32(w)
    assert np.array_equal(mine, bs)
