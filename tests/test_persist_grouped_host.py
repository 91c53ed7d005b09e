"""Host-side checks of the persisted-weight header and of the grouped-scale oracle (no GPU needed).

- The restated grouped accumulate (oracle/ork_oracle.c orc_gemm_grouped) equals ork-driver's own
  orki_cpu_gemm_grouped (src/npu/core/buf.c:501-520) and its offline ork_i4_mm_run_grouped /
  ork_i8_mm_run_grouped paths (after ork_i4_mm_pack_grouped, or ork_i4_w_dump_cpu + ork_i4a8_mm_load_tiled)
  bit for bit, compiled from the reference's sources (oracle/_ref).
- The header this library stamps has the reference's layout (src/npu/core/packhdr.c, include/ork/weights.h:
  180-198): same magic, format, dtype, K, N, header size and zero padding, only the caps id and device id
  differ -- and each build refuses the other's blob with ORK_PACKERR_CAPS.
- ork_b200_pack_check reports the reference's refusal codes in the reference's order.
"""
import ctypes as C
import struct

import numpy as np
import pytest

import oracle_ffi as of
import ork_b200

_p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
PACKERR = {"short": -1, "unstamped": -2, "format": -3, "caps": -4, "shape": -5}
HDR = 4096


def _ref():
    r = of.reference()
    if r is None:
        pytest.skip("oracle/_ref not built (the reference sources are not present)")
    return r


def _case(seed, M, K, N, G, a_lo=-128, a_hi=128):
    rng = np.random.default_rng(seed)
    A = rng.integers(a_lo, a_hi, size=(M, K), dtype=np.int8)
    B = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    aS = rng.uniform(1e-3, 2e-2, size=(M, K // G)).astype(np.float32)
    bS = rng.uniform(1e-3, 2e-2, size=(K // G, N)).astype(np.float32)
    return A, B, aS, bS


@pytest.mark.parametrize("M,K,N,G", [(1, 256, 64, 32), (5, 512, 128, 128), (3, 1024, 192, 256), (2, 384, 64, 384)])
def test_grouped_oracle_equals_reference_kernel(M, K, N, G):
    ref = _ref()
    A, B, aS, bS = _case(M * 7 + G, M, K, N, G)
    want = np.empty((M, N), np.float32)
    assert ref.orki_cpu_gemm_grouped(M, K, N, G, _p(A), _p(B), _p(aS), _p(bS), _p(want)) == 0
    got = of.gemm_grouped(A, B, G, aS, bS)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("M,K,N,G", [(4, 512, 128, 64), (1, 1024, 64, 1024)])
def test_grouped_oracle_equals_reference_offline_runs(M, K, N, G):
    """The reference's offline W4A4 grouped pack+run and its tiled-load int8 grouped run."""
    ref = _ref()
    ctx = ref.ork_npu_init_offline(b"rk3588")
    assert ctx
    try:
        A4, B, aS, bS = _case(G + M, M, K, N, G, -8, 8)
        w = ref.ork_i4_mm_pack_grouped(ctx, K, N, _p(B), G)
        assert w
        C4 = np.empty((M, N), np.float32)
        assert ref.ork_i4_mm_run_grouped(ctx, w, M, _p(A4), _p(aS), _p(bS), _p(C4)) == 0
        ref.ork_w_free(w)
        assert np.array_equal(C4.view(np.uint32), of.gemm_grouped(A4, B, G, aS, bS).view(np.uint32))

        need = ref.ork_i4_w_dump_cpu(ctx, K, N, _p(B), None, 0)
        blob = np.zeros(need, np.uint8)
        assert ref.ork_i4_w_dump_cpu(ctx, K, N, _p(B), _p(blob), need) == need
        wt = ref.ork_i4a8_mm_load_tiled(ctx, K, N, _p(blob), need, G)
        assert wt
        A8 = np.random.default_rng(3).integers(-128, 128, size=(M, K), dtype=np.int8)
        # the reference's offline tiled load keeps codes only; the group size is attached afterwards
        ref.ork_w_set_group.restype = C.c_int
        ref.ork_w_set_group.argtypes = [C.c_void_p, C.c_int]
        assert ref.ork_w_set_group(wt, G) == 0
        C8 = np.empty((M, N), np.float32)
        assert ref.ork_i8_mm_run_grouped(ctx, wt, M, _p(A8), _p(aS), _p(bS), _p(C8)) == 0
        ref.ork_w_free(wt)
        assert np.array_equal(C8.view(np.uint32), of.gemm_grouped(A8, B, G, aS, bS).view(np.uint32))
    finally:
        ref.ork_npu_free(ctx)


def _hdr(blob):
    magic, fmt, capid, dtype, K, N, hb, flags = struct.unpack_from("<IIIIiiII", bytes(blob[:32]))
    soc = bytes(blob[32:48]).split(b"\0")[0].decode()
    return dict(magic=magic, fmt=fmt, capid=capid, dtype=dtype, K=K, N=N, hdr_bytes=hb, flags=flags, soc=soc)


@pytest.mark.parametrize("kind", ["i8", "i4"])
def test_header_layout_matches_reference_and_builds_refuse_each_other(kind):
    ref = _ref()
    L = ork_b200.lib()
    K, N = 256, 128
    B = np.random.default_rng(1).integers(-8, 8, size=(K, N), dtype=np.int8)
    dtype = 1 if kind == "i8" else 2
    ours_fn = L.ork_i8_w_dump_cpu if kind == "i8" else L.ork_i4_w_dump_cpu
    ref_fn = ref.ork_i8_w_dump_cpu if kind == "i8" else ref.ork_i4_w_dump_cpu
    need = ours_fn(None, K, N, _p(B), None, 0)
    ours = np.zeros(need, np.uint8)
    assert ours_fn(None, K, N, _p(B), _p(ours), need) == need
    ctx = ref.ork_npu_init_offline(b"rk3588")
    try:
        rneed = ref_fn(ctx, K, N, _p(B), None, 0)
        theirs = np.zeros(rneed, np.uint8)
        assert ref_fn(ctx, K, N, _p(B), _p(theirs), rneed) == rneed
        h_o, h_t = _hdr(ours), _hdr(theirs)
        for f in ("magic", "fmt", "dtype", "K", "N", "hdr_bytes", "flags"):
            assert h_o[f] == h_t[f], f
        assert h_o["magic"] == 0x4B50414F and h_o["hdr_bytes"] == HDR and h_o["dtype"] == dtype
        assert h_o["soc"] == "b200" and h_t["soc"] == "rk3588"
        assert h_o["capid"] == L.ork_b200_pack_capid() and h_o["capid"] != h_t["capid"]
        assert not ours[48:HDR].any() and not theirs[48:HDR].any()  # zero padding on both sides
        assert L.ork_pack_hdr_bytes() == HDR
        # each build refuses the other's tiles: same shape and dtype, different caps
        assert L.ork_b200_pack_check(_p(theirs), rneed, dtype, K, N) == PACKERR["caps"]
        assert ref.orki_pack_check(ctx, _p(ours), need, dtype, K, N) == PACKERR["caps"]
        assert L.ork_b200_pack_check(_p(ours), need, dtype, K, N) == 0
        assert ref.orki_pack_check(ctx, _p(theirs), rneed, dtype, K, N) == 0
    finally:
        ref.ork_npu_free(ctx)


def test_pack_check_codes_in_reference_order():
    L = ork_b200.lib()
    K, N = 64, 64
    B = np.ones((K, N), np.int8)
    need = L.ork_i8_w_dump_cpu(None, K, N, _p(B), None, 0)
    assert need == HDR + K * N
    good = np.zeros(need, np.uint8)
    assert L.ork_i8_w_dump_cpu(None, K, N, _p(B), _p(good), need) == need
    assert L.ork_i8_w_dump_cpu(None, K, N, _p(B), _p(good), need - 1) == 0  # short cap
    assert np.array_equal(good[HDR:], np.ones(K * N, np.uint8))  # payload: codes [N][K]
    chk = lambda b, n=None, dt=1, k=K, nn=N: L.ork_b200_pack_check(_p(b), len(b) if n is None else n, dt, k, nn)  # noqa
    assert chk(good) == 0
    assert chk(good, HDR - 1) == PACKERR["short"]
    bad = good.copy(); bad[0] ^= 1
    assert chk(bad) == PACKERR["unstamped"]
    bad = good.copy(); bad[4] ^= 2  # fmt
    assert chk(bad) == PACKERR["format"]
    bad = good.copy(); bad[8] ^= 1  # capid
    assert chk(bad) == PACKERR["caps"]
    bad = good.copy(); bad[24] ^= 1  # hdr_bytes
    assert chk(bad) == PACKERR["format"]
    assert chk(good, dt=2) == PACKERR["shape"]
    assert chk(good, k=K + 32) == PACKERR["shape"]
    assert chk(good, nn=N + 32) == PACKERR["shape"]
    # unstamped wins over every later cause, format over caps (the reference's order)
    bad = good.copy(); bad[0] ^= 1; bad[8] ^= 1
    assert chk(bad, dt=2) == PACKERR["unstamped"]
    bad = good.copy(); bad[4] ^= 2; bad[8] ^= 1
    assert chk(bad) == PACKERR["format"]


def test_i4_dump_cpu_payload_is_w4a4_nibbles():
    L = ork_b200.lib()
    K, N = 64, 128
    B = np.random.default_rng(2).integers(-8, 8, size=(K, N), dtype=np.int8)
    need = L.ork_i4_w_dump_cpu(None, K, N, _p(B), None, 0)
    assert need == HDR + K * N // 2
    blob = np.zeros(need, np.uint8)
    assert L.ork_i4_w_dump_cpu(None, K, N, _p(B), _p(blob), need) == need
    nib = blob[HDR:].reshape(N, K // 2)
    lo, hi = (nib & 15).astype(np.int16), (nib >> 4).astype(np.int16)
    codes = np.empty((N, K), np.int16)
    codes[:, 0::2], codes[:, 1::2] = lo, hi
    codes[codes >= 8] -= 16
    assert np.array_equal(codes, B.T.astype(np.int16))
    assert L.ork_i4_w_dump_cpu(None, K, 96, _p(B), None, 0) == 0  # N % 64
    assert L.ork_i8_w_dump_bf_cpu(None, K, N, _p(B), None, 0) == 0  # no full-K companion layout


def test_restated_grouped_reproduces_reference_fixtures():
    """The restated oracle against the fp32 results recorded from the reference (no reference tree needed)."""
    import hashlib
    import json
    import os

    from make_fixtures import grouped_inputs

    fx = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_fixtures.json")))["grouped"]
    assert len(fx) >= 4
    for name, c in fx.items():
        A, B, aS, bS = grouped_inputs(c["seed"], c["M"], c["K"], c["N"], c["G"], c["a_range"])
        got = of.gemm_grouped(A, B, c["G"], aS, bS)
        assert hashlib.sha256(got.tobytes()).hexdigest() == c["c_sha256"], name
