"""ctypes access to the parity checkers under oracle/ (test infrastructure only).

- `restated()`   -> oracle/liborkoracle.so : the C restatement of the reference path (ork_oracle.c).
- `reference()`  -> oracle/_ref/libork_ref.so : ork-driver's own CPU code, compiled from its sources by
  oracle/Makefile (present only where the reference tree was available at build time), or None.

Also the reference example tests' fixed-seed input generators (examples/quant.c:18,
examples/test_matmul.c:11), so the goldens those tests hard-code can be reproduced on identical inputs.
"""
import ctypes as C
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(ROOT, "oracle")
_restated = None
_reference = None

FNV_OFFSET = 1469598103934665603

_p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731


def restated():
    global _restated
    if _restated is None:
        path = os.path.join(ORACLE_DIR, "liborkoracle.so")
        lib = C.CDLL(path)
        lib.orc_fnv64.restype = C.c_uint64
        lib.orc_fnv64.argtypes = [C.c_uint64, C.c_void_p, C.c_size_t]
        lib.orc_lcg_skip.restype = C.c_uint32
        lib.orc_lcg_skip.argtypes = [C.c_uint32, C.c_uint64]
        lib.orc_i4a8_blob.restype = C.c_size_t
        lib.orc_i4a8_blob.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                      C.c_void_p, C.c_size_t]
        lib.orc_i4a8_blob_codes.restype = C.c_int
        lib.orc_i4a8_blob_codes.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_size_t, C.c_void_p,
                                            C.c_void_p, C.c_void_p]
        for name in ("orc_gemm_i32", "orc_gemm_i32_nk", "orc_gemm_f16"):
            getattr(lib, name).argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        lib.orc_i8_quant_f32.argtypes = [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        lib.orc_gen_frand.argtypes = [C.POINTER(C.c_uint32), C.c_void_p, C.c_size_t]
        lib.orc_gen_rnd_i8.argtypes = [C.POINTER(C.c_uint32), C.c_void_p, C.c_size_t, C.c_int]
        lib.orc_gen_rnd_f16.argtypes = [C.POINTER(C.c_uint32), C.c_void_p, C.c_size_t]
        lib.orc_nf4_lut.argtypes = [C.c_void_p]
        lib.orc_threads.restype = C.c_int
        lib.orc_set_threads.restype = C.c_int
        lib.orc_set_threads.argtypes = [C.c_int]
        lib.orc_swiglu_q8.restype = C.c_float
        lib.orc_swiglu_q8.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_void_p]
        lib.orc_rms_q8.restype = C.c_float
        lib.orc_rms_q8.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        lib.orc_layer_i8.restype = C.c_int
        lib.orc_layer_i8.argtypes = [C.c_void_p, C.c_double, C.c_double] + [C.c_void_p] * 7 + [C.c_void_p] * 7 + \
            [C.c_int, C.c_void_p, C.c_int]
        lib.orc_gemm_grouped.restype = C.c_int
        lib.orc_requant.argtypes = [C.c_size_t, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]
        lib.orc_requant.restype = None
        lib.orc_gemm_grouped.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_void_p, C.c_void_p]
        _restated = lib
    return _restated


def reference():
    """The reference's compiled CPU code, or None when oracle/_ref was not built."""
    global _reference
    if _reference is None:
        path = os.path.join(ORACLE_DIR, "_ref", "libork_ref.so")
        if not os.path.exists(path):
            return None
        lib = C.CDLL(path)
        lib.ork_npu_init_offline.restype = C.c_void_p
        lib.ork_npu_init_offline.argtypes = [C.c_char_p]
        lib.ork_npu_free.argtypes = [C.c_void_p]
        lib.ork_i8_mm_pack.restype = C.c_void_p
        lib.ork_i8_mm_pack.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        lib.ork_i4_mm_pack.restype = C.c_void_p
        lib.ork_i4_mm_pack.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        for name in ("ork_i8_mm_run", "ork_i4_mm_run"):
            getattr(lib, name).restype = C.c_int
            getattr(lib, name).argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        lib.ork_i4a8_pack_cpu_blob_qerr.restype = C.c_size_t
        lib.ork_i4a8_pack_cpu_blob_qerr.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                                    C.c_int, C.c_void_p, C.c_size_t, C.c_void_p]
        lib.ork_i4a8_mm_load.restype = C.c_void_p
        lib.ork_i4a8_mm_load.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]
        lib.ork_w_bscale.restype = C.POINTER(C.c_float)
        lib.ork_w_bscale.argtypes = [C.c_void_p]
        lib.ork_w_quant_kind.restype = C.c_int
        lib.ork_w_quant_kind.argtypes = [C.c_void_p]
        lib.ork_w_codes.restype = C.POINTER(C.c_int8)
        lib.ork_w_codes.argtypes = [C.c_void_p]
        lib.ork_w_free.argtypes = [C.c_void_p]
        lib.ork_i8_mm_run_cpu.argtypes = [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        # grouped scales (src/npu/core/buf.c:501, src/npu/i4/pack.c:686, src/npu/i4/run.c:367,
        # src/npu/i4/pack.c:265, src/npu/i8/run.c:45) and the persisted-weight header (src/npu/core/packhdr.c)
        lib.orki_cpu_gemm_grouped.restype = C.c_int
        lib.orki_cpu_gemm_grouped.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                              C.c_void_p, C.c_void_p, C.c_void_p]
        lib.ork_i4_mm_pack_grouped.restype = C.c_void_p
        lib.ork_i4_mm_pack_grouped.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int]
        for name in ("ork_i4_mm_run_grouped", "ork_i8_mm_run_grouped"):
            getattr(lib, name).restype = C.c_int
            getattr(lib, name).argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_void_p]
        for name in ("ork_i8_w_dump_cpu", "ork_i4_w_dump_cpu"):
            getattr(lib, name).restype = C.c_size_t
            getattr(lib, name).argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_size_t]
        lib.ork_i4a8_mm_load_tiled.restype = C.c_void_p
        lib.ork_i4a8_mm_load_tiled.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t, C.c_int]
        lib.orki_pack_check.restype = C.c_int
        lib.orki_pack_check.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_int]
        lib.ref_layer_i8.restype = C.c_int
        lib.ref_layer_i8.argtypes = [C.c_void_p, C.c_double, C.c_double] + [C.c_void_p] * 7 + [C.c_void_p] * 7
        lib.orki_pack_capid.restype = C.c_uint
        lib.orki_pack_capid.argtypes = [C.c_void_p]
        _reference = lib
    return _reference


# --------------------------------------------------------------------------------------------------
# thin numpy wrappers over the restatement

def fnv64(arr, h=FNV_OFFSET):
    a = np.ascontiguousarray(arr)
    return restated().orc_fnv64(h, _p(a), a.nbytes)


def gemm_i32(A, B_kn):
    """C = A[M,K] . B[K,N] exactly in int32 (src/npu/core/buf.c:428)."""
    A = np.ascontiguousarray(A, np.int8)
    B_kn = np.ascontiguousarray(B_kn, np.int8)
    M, K = A.shape
    N = B_kn.shape[1]
    Cm = np.empty((M, N), np.int32)
    restated().orc_gemm_i32(M, K, N, _p(A), _p(B_kn), _p(Cm))
    return Cm


def gemm_i32_nk(A, Bt_nk):
    A = np.ascontiguousarray(A, np.int8)
    Bt_nk = np.ascontiguousarray(Bt_nk, np.int8)
    M, K = A.shape
    N = Bt_nk.shape[0]
    Cm = np.empty((M, N), np.int32)
    restated().orc_gemm_i32_nk(M, K, N, _p(A), _p(Bt_nk), _p(Cm))
    return Cm


def gemm_f16(A, B_kn):
    """Sequential-f32 reference of examples/test_matmul.c:37 on float16 inputs."""
    A = np.ascontiguousarray(A, np.float16)
    B_kn = np.ascontiguousarray(B_kn, np.float16)
    M, K = A.shape
    N = B_kn.shape[1]
    Cm = np.empty((M, N), np.float32)
    restated().orc_gemm_f16(M, K, N, _p(A), _p(B_kn), _p(Cm))
    return Cm


def gemm_grouped(A, B_kn, G, aS, bS):
    """C fp32 = sum over K-groups of ((float)int32 dot * aS[m][g]) * bS[g][n], g ascending
    (src/npu/core/buf.c:501-520)."""
    A = np.ascontiguousarray(A, np.int8)
    B_kn = np.ascontiguousarray(B_kn, np.int8)
    aS = np.ascontiguousarray(aS, np.float32)
    bS = np.ascontiguousarray(bS, np.float32)
    M, K = A.shape
    N = B_kn.shape[1]
    Cm = np.empty((M, N), np.float32)
    assert restated().orc_gemm_grouped(M, K, N, G, _p(A), _p(B_kn), _p(aS), _p(bS), _p(Cm)) == 0
    return Cm


LAYER_KEYS = ("D", "H", "Hkv", "dk", "dv", "Nff", "nkv", "pos")


def layer_inputs(seed, D, H, Hkv, dk, Nff, nkv, pos, hstride=None):
    """Seeded inputs of one decode layer: weight codes B [K][N] (q, k, v, o, gate, up, down), norm gains,
    x, and K/V caches [Hkv][hstride][dk] (hstride >= nkv + 1 leaves room for the token's own k/v)."""
    rng = np.random.default_rng(seed)
    Nq, Nk = H * dk, Hkv * dk
    shapes = [(D, Nq), (D, Nk), (D, Nk), (Nq, D), (D, Nff), (D, Nff), (Nff, D)]
    Bs = [rng.integers(-127, 128, size=s, dtype=np.int8) for s in shapes]
    norms = [rng.uniform(0.5, 1.5, size=n).astype(np.float32) for n in (D, dk, D, dk)]  # attn, q, ffn, k
    x = rng.standard_normal(D).astype(np.float32)
    hs = hstride or nkv
    Kc = np.zeros((Hkv, hs, dk), np.float32)
    Vc = np.zeros((Hkv, hs, dk), np.float32)
    Kc[:, :nkv] = rng.standard_normal((Hkv, nkv, dk)).astype(np.float32)
    Vc[:, :nkv] = rng.standard_normal((Hkv, nkv, dk)).astype(np.float32)
    return Bs, norms, x, Kc, Vc


def layer(dims, attn_scale, rope_base, Bs, norms, x, Kc, Vc, kv_ext=False, hstride=0, k_norm=True):
    """The restated decode layer (src/npu/i8/chain.c:106-122); with kv_ext the token's k/v are written into
    copies of the caches at slot nkv first. Returns (x_out, Kc, Vc)."""
    dm = np.array([dims[k] for k in LAYER_KEYS], np.uint32)
    Kc, Vc = Kc.copy(), Vc.copy()
    out = np.zeros(dims["D"], np.float32)
    Bs = [np.ascontiguousarray(b) for b in Bs]
    kn = norms[3] if k_norm else None
    rc = restated().orc_layer_i8(_p(dm), attn_scale, rope_base, *[_p(b) for b in Bs], _p(norms[0]), _p(norms[1]),
                                 _p(norms[2]), _p(x), _p(Kc), _p(Vc), _p(out), int(kv_ext),
                                 None if kn is None else _p(kn), hstride)
    assert rc == 0
    return out, Kc, Vc


def rms_q8(x, g=None):
    """RMSNorm + per-tensor int8 quantization of one row (src/spine_kernels.h spine_rmsnorm + spine_quant):
    (codes int8 [n], scale s)."""
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.size, np.int8)
    s = restated().orc_rms_q8(_p(x), None if g is None else _p(np.ascontiguousarray(g, np.float32)), x.size, _p(q))
    return q, s


def swiglu_q8(cg, cu, s):
    """The decode layer's FFN epilogue over one row (spine_silu_glu + spine_quant): (codes int8 [n], scale)."""
    cg = np.ascontiguousarray(cg, np.int32)
    cu = np.ascontiguousarray(cu, np.int32)
    q = np.empty(cg.size, np.int8)
    sh = restated().orc_swiglu_q8(_p(cg), _p(cu), cg.size, float(s), _p(q))
    return q, sh


def i8_quant_f32(f32_nk):
    """Codes [N][K] and bscale[N] of ork_i8_mm_pack_f32 (src/npu.c:854, src/npu/i8/pack.c:450)."""
    f32_nk = np.ascontiguousarray(f32_nk, np.float32)
    N, K = f32_nk.shape
    codes = np.empty((N, K), np.int8)
    bs = np.empty(N, np.float32)
    restated().orc_i8_quant_f32(K, N, _p(f32_nk), _p(codes), _p(bs))
    return codes, bs


def i4a8_blob(f32_nk, imatrix=None, nf4=False, sr=False):
    f32_nk = np.ascontiguousarray(f32_nk, np.float32)
    N, K = f32_nk.shape
    lib = restated()
    need = lib.orc_i4a8_blob(K, N, _p(f32_nk), None, int(nf4), int(sr), None, 0)
    out = np.zeros(need, np.uint8)
    im = None if imatrix is None else np.ascontiguousarray(imatrix, np.float32)
    got = lib.orc_i4a8_blob(K, N, _p(f32_nk), None if im is None else _p(im), int(nf4), int(sr), _p(out), need)
    assert got == need
    return out


def i4a8_blob_codes(blob, K, N):
    """(codes [K][N] int8, bscale[N], quant_kind) of an O4N1 blob, or None if the blob is refused."""
    blob = np.ascontiguousarray(blob, np.uint8)
    codes = np.empty((K, N), np.int8)
    bs = np.empty(N, np.float32)
    qk = C.c_int(-1)
    rc = restated().orc_i4a8_blob_codes(K, N, _p(blob), blob.nbytes, _p(codes), _p(bs), C.byref(qk))
    if rc != 0:
        return None
    return codes, bs, qk.value


def nf4_lut():
    lut = np.empty(16, np.int8)
    restated().orc_nf4_lut(_p(lut))
    return lut


class Lcg:
    """The example tests' LCG (sd = sd*1103515245 + 12345), with their two output mappings."""

    def __init__(self, seed):
        self.sd = C.c_uint32(seed)

    def frand(self, n):  # examples/quant.c:18
        out = np.empty(n, np.float32)
        restated().orc_gen_frand(C.byref(self.sd), _p(out), n)
        return out

    def rnd_i8(self, n, offset=1):  # examples/test_matmul.c:11, used as (int8_t)(rnd()-1)
        out = np.empty(n, np.int8)
        restated().orc_gen_rnd_i8(C.byref(self.sd), _p(out), n, offset)
        return out

    def rnd_f16(self, n):  # examples/test_matmul.c:23-24, (f16)rnd()
        out = np.empty(n, np.uint16)
        restated().orc_gen_rnd_f16(C.byref(self.sd), _p(out), n)
        return out.view(np.float16)

    def skip(self, n):
        self.sd = C.c_uint32(restated().orc_lcg_skip(self.sd.value, n))


def requant(acc, mult, shift, bits=8, g=None):
    """The fused output stage on int32 sums (optionally times g first): the reference's requant model
    (examples/test_mm_i8_out8.c:24-33), restated in oracle/ork_oracle.c."""
    acc = np.ascontiguousarray(acc, np.int32)
    out = np.empty(acc.shape, np.int16 if bits == 16 else np.int8)
    gp = None
    if g is not None:
        g = np.ascontiguousarray(g, np.int8)
        assert g.shape == acc.shape
        gp = _p(g)
    restated().orc_requant(acc.size, _p(acc), gp, int(mult), int(shift), bits, _p(out))
    return out
