"""The drop-in boundary, checked without a GPU: libork_npu.so loads, exports every function that
include/*.h declares (and nothing else), and the calls that need no device behave like the reference's
(NULL / -1 / 0 on bad arguments, the version tokens, the host-only O4N1 writer)."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

import ork_b200

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in ("ork_npu.h", "ork_b200.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"\b(ork_[a-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_exactly_the_declared_functions():
    out = subprocess.run(["nm", "-D", "--defined-only", ork_b200.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    declared = declared_functions()
    assert declared, "no declarations parsed"
    assert declared <= exported, sorted(declared - exported)
    assert {e for e in exported if e.startswith("ork_")} == declared, sorted(exported - declared)


def test_binding_covers_every_declared_function():
    assert {n for n, _, _ in ork_b200.SIGNATURES} == declared_functions()
    ork_b200.lib()  # every prototype resolves


def test_version_tokens():
    L = ork_b200.lib()
    assert L.ork_npu_version().decode().startswith("1.0.190")
    assert L.ork_pack_format_version() == 1


def test_null_and_bad_argument_conventions():
    L = ork_b200.lib()
    B = np.zeros((32, 32), np.int8)
    f = np.zeros((32, 32), np.float32)
    # pack / load on a NULL context -> NULL (bad dims would too)
    assert not L.ork_i8_mm_pack(None, 32, 32, B.ctypes.data)
    assert not L.ork_i8_mm_pack_f32(None, 32, 32, f.ctypes.data, None)
    assert not L.ork_i4a8_mm_pack(None, 32, 32, f.ctypes.data, None)
    assert not L.ork_i4_mm_pack(None, 32, 64, B.ctypes.data)
    assert not L.ork_f16_mm_pack(None, 32, 16, B.ctypes.data)
    assert not L.ork_i4a8_mm_load(None, 32, 32, B.ctypes.data, 100)
    # run with NULLs -> -1
    assert L.ork_i8_mm_run(None, None, 1, None, None) == -1
    assert L.ork_i4_mm_run(None, None, 1, None, None) == -1
    assert L.ork_f16_mm_run(None, None, 1, None, None) == -1
    # accessors on NULL (include/ork/weights.h:154-158)
    k, n = C.c_int(7), C.c_int(7)
    L.ork_w_dims(None, C.byref(k), C.byref(n))
    assert (k.value, n.value) == (0, 0)
    assert L.ork_w_quant_kind(None) == -1
    assert not L.ork_w_bscale(None)
    assert L.ork_i4a8_w_dump(None, None, 0) == 0
    assert L.ork_w_bytes(None) == 0
    L.ork_w_free(None)
    L.ork_mm_free(None, None)
    L.ork_npu_free(None)


@pytest.mark.parametrize("K,N", [(31, 32), (32, 31), (0, 32), (32, 0), (48, 32)])
def test_cpu_blob_refuses_bad_dims(K, N):
    L = ork_b200.lib()
    f = np.zeros(max(1, K * N), np.float32)
    assert L.ork_i4a8_pack_cpu_blob(None, K, N, f.ctypes.data, None, 0, None, 0) == 0


def test_cpu_blob_size_query_and_short_cap():
    L = ork_b200.lib()
    K, N = 64, 32
    f = np.ones((N, K), np.float32)
    need = L.ork_i4a8_pack_cpu_blob(None, K, N, f.ctypes.data, None, 0, None, 0)
    assert need == 20 + 4 * N + K * N // 2
    out = np.zeros(need, np.uint8)
    assert L.ork_i4a8_pack_cpu_blob(None, K, N, f.ctypes.data, None, 0, out.ctypes.data, need - 1) == 0
    assert L.ork_i4a8_pack_cpu_blob(None, K, N, f.ctypes.data, None, 0, out.ctypes.data, need) == need


def test_init_without_gpu_returns_null():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert not ork_b200.lib().ork_npu_init()


def test_cpu_matmul_entry_is_exact():
    from oracle_ffi import gemm_i32

    rng = np.random.default_rng(0)
    A = rng.integers(-128, 128, size=(5, 96), dtype=np.int8)
    B = rng.integers(-128, 128, size=(96, 64), dtype=np.int8)
    Cm = np.zeros((5, 64), np.int32)
    ork_b200.lib().ork_i8_mm_run_cpu(5, 96, 64, A.ctypes.data, B.ctypes.data, Cm.ctypes.data)
    assert np.array_equal(Cm, gemm_i32(A, B))


def _exported():
    out = subprocess.run(["nm", "-D", "--defined-only", ork_b200.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln and ln.split()[-1].startswith("ork_")}


def test_shared_names_have_the_reference_prototypes():
    """A caller that binds a symbol by its ork-driver name (a ggml-ork backend, an FFI table) must get the
    reference's function: every exported name that ork-driver's public headers also declare has exactly
    the reference's return and parameter types (tests/golden/reference_prototypes.json, written from the
    reference's include/ork_npu.h and include/ork/*.h by tests/golden/make_reference_prototypes.py)."""
    import json

    from cproto import prototypes

    ref = json.load(open(os.path.join(ROOT, "tests", "golden", "reference_prototypes.json")))["prototypes"]
    ours = prototypes([open(os.path.join(ROOT, "include", h)).read() for h in ("ork_npu.h", "ork_b200.h")])
    shared = sorted(_exported() & set(ref))
    assert len(shared) >= 50, shared
    bad = {n: (ours.get(n), ref[n]) for n in shared if ours.get(n) != ref[n]}
    assert not bad, bad


def test_b200_additions_are_prefixed():
    """Names this library adds beyond the reference's API live under ork_b200_ (ork_i8_mm_run_noalloc, an
    addition the reference has no name for either, is the one exception), so no future or unread part
    of the reference's API can collide with them."""
    import json

    ref = json.load(open(os.path.join(ROOT, "tests", "golden", "reference_prototypes.json")))["prototypes"]
    extra = sorted(n for n in _exported() - set(ref) if not n.startswith("ork_b200_"))
    assert extra == ["ork_i8_mm_run_noalloc"], extra


def test_async_launchers_refuse_like_the_reference():
    """The ork_async launchers' NULL refusals (src/npu.c:2212-2222, src/npu/i8/run.c:778-784) and
    ork_async_wait(NULL) == -1, without a device."""
    L = ork_b200.lib()
    for fn in (L.ork_mm_run_async, L.ork_i8_mm_run_async, L.ork_i4_mm_run_async):
        assert not fn(None, None, 1, None, None)
    for fn in (L.ork_i8_mm_run_chain_async, L.ork_i4_mm_run_chain_async, L.ork_i8_mm_run_stream_async,
               L.ork_i4_mm_run_stream_async):
        assert not fn(None, 1, None)
    assert L.ork_async_wait(None) == -1
    assert L.ork_npu_last_async_cpu(None) == -1
    assert L.ork_i4_mm_run_stream(None, 1, None) == -1
    assert L.ork_b200_reload_tuning(None) == -1
