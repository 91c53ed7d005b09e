"""ctypes binding of libork_npu.so (include/ork_npu.h + include/ork_b200.h).

Mirrors the reference's C API one to one (same function names, argument order and return codes), with
thin numpy helpers on top so tests and benchmarks read like ork-driver's own examples/*.c checks. The
library is loaded from this directory; there is no fallback of any kind: if libork_npu.so is missing
this module raises on import of `lib()`.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libork_npu.so")

ORK_QK_UNIFORM = 0
ORK_QK_CODEBOOK_NF4 = 1

_lib = None

# (name, restype, argtypes) for every function declared in include/ork_npu.h and include/ork_b200.h.
_vp, _i, _sz, _f = C.c_void_p, C.c_int, C.c_size_t, C.c_float
SIGNATURES = [
    ("ork_npu_version", C.c_char_p, []),
    ("ork_pack_format_version", C.c_uint32, []),
    ("ork_npu_init", _vp, []),
    ("ork_npu_free", None, [_vp]),
    ("ork_f16_mm_pack", _vp, [_vp, _i, _i, _vp]),
    ("ork_i8_mm_pack", _vp, [_vp, _i, _i, _vp]),
    ("ork_i8_mm_pack_f32", _vp, [_vp, _i, _i, _vp, _vp]),
    ("ork_i4a8_mm_pack", _vp, [_vp, _i, _i, _vp, _vp]),
    ("ork_i4a8_mm_pack_im", _vp, [_vp, _i, _i, _vp, _vp, _vp]),
    ("ork_i4_mm_pack", _vp, [_vp, _i, _i, _vp]),
    ("ork_i4a8_w_dump", _sz, [_vp, _vp, _sz]),
    ("ork_i4a8_mm_load", _vp, [_vp, _i, _i, _vp, _sz]),
    ("ork_i4a8_pack_cpu_blob", _sz, [_vp, _i, _i, _vp, _vp, _i, _vp, _sz]),
    ("ork_i4a8_pack_cpu_blob_qerr", _sz, [_vp, _i, _i, _vp, _vp, _i, _vp, _sz, C.POINTER(_f)]),
    ("ork_w_free", None, [_vp]),
    ("ork_mm_free", None, [_vp, _vp]),
    ("ork_w_bytes", _sz, [_vp]),
    ("ork_w_dims", None, [_vp, C.POINTER(_i), C.POINTER(_i)]),
    ("ork_w_quant_kind", _i, [_vp]),
    ("ork_w_bscale", C.POINTER(_f), [_vp]),
    ("ork_f16_mm_run", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_i8_mm_run", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_i4_mm_run", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_i8_mm_run_cpu", None, [_i, _i, _i, _vp, _vp, _vp]),
    ("ork_b200_i8_mm_run_async", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_i8_mm_run_out8", _i, [_vp, _vp, _i, _vp, _vp, _i, _i]),
    ("ork_i8_mm_run_out16", _i, [_vp, _vp, _i, _vp, _vp, _i, _i]),
    ("ork_i8_mm_run_ewmul", _i, [_vp, _vp, _i, _vp, _vp, _vp, _i, _i]),
    ("ork_b200_i8_mm_run_out8_async", _i, [_vp, _vp, _i, _vp, _vp, _i, _i]),
    ("ork_b200_i8_mm_run_out16_async", _i, [_vp, _vp, _i, _vp, _vp, _i, _i]),
    ("ork_b200_i8_mm_run_ewmul_async", _i, [_vp, _vp, _i, _vp, _vp, _vp, _i, _i]),
    ("ork_i8_npu_ewmul", _i, [_vp, _vp, _vp, _i, _i, _i, _i, _vp, C.POINTER(C.c_double)]),
    ("ork_b200_sym_alloc", _vp, [_vp, _sz, _vp]),
    ("ork_b200_sym_free", _i, [_vp, _vp]),
    ("ork_b200_sym_open", _vp, [_vp, _vp]),
    ("ork_b200_sym_close", _i, [_vp, _vp]),
    ("ork_b200_peers_create", _vp, [_vp, _i, _i, C.POINTER(_vp), C.POINTER(_vp), _i, _i, _i]),
    ("ork_b200_peers_destroy", None, [_vp]),
    ("ork_b200_i8_mm_run_peers_async", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_b200_i4_mm_run_peers_async", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_b200_peers_wait_async", _i, [_vp, _vp]),
    ("ork_b200_i8_mm_run_gather_async", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_b200_i4_mm_run_gather_async", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_b200_peers_land", _i, [_vp, C.POINTER(_vp), _i]),
    ("ork_b200_copy", _i, [_vp, _vp, _vp, _sz]),
    ("ork_b200_i4_mm_run_async", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_b200_f16_mm_run_async", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_i8_mm_run_noalloc", _i, [_vp, _vp, _i, _vp, _vp]),
    ("ork_pack_hdr_bytes", _sz, []),
    ("ork_w_dump", _sz, [_vp, _vp, _sz]),
    ("ork_i8_w_dump_cpu", _sz, [_vp, _i, _i, _vp, _vp, _sz]),
    ("ork_i8_w_dump_bf_cpu", _sz, [_vp, _i, _i, _vp, _vp, _sz]),
    ("ork_i4_w_dump_cpu", _sz, [_vp, _i, _i, _vp, _vp, _sz]),
    ("ork_f16_mm_load", _vp, [_vp, _i, _i, _vp, _sz]),
    ("ork_i8_mm_load", _vp, [_vp, _i, _i, _vp, _sz]),
    ("ork_i4_mm_load", _vp, [_vp, _i, _i, _vp, _sz]),
    ("ork_i4a8_mm_load_tiled", _vp, [_vp, _i, _i, _vp, _sz, _i]),
    ("ork_i4_mm_pack_grouped", _vp, [_vp, _i, _i, _vp, _i]),
    ("ork_w_set_group", _i, [_vp, _i]),
    ("ork_i4_mm_run_grouped", _i, [_vp, _vp, _i, _vp, _vp, _vp, _vp]),
    ("ork_i8_mm_run_grouped", _i, [_vp, _vp, _i, _vp, _vp, _vp, _vp]),
    ("ork_b200_i4_mm_run_grouped_async", _i, [_vp, _vp, _i, _vp, _vp, _vp, _vp]),
    ("ork_b200_i8_mm_run_grouped_async", _i, [_vp, _vp, _i, _vp, _vp, _vp, _vp]),
    ("ork_i8_mm_run_chain", _i, [_vp, _i, _vp]),
    ("ork_i8_mm_run_stream", _i, [_vp, _i, _vp]),
    ("ork_b200_i8_mm_run_chain_async", _i, [_vp, _i, _vp]),
    ("ork_i4_mm_run_chain", _i, [_vp, _i, _vp]),
    ("ork_i4_mm_run_experts", _i, [_vp, _vp, _i, _i]),
    ("ork_mm_submit", _i, [_vp, _vp, _i, _vp]),
    ("ork_mm_collect", _i, [_vp, _i, _vp]),
    ("ork_i8_mm_layer", _i, [_vp, _vp] + [_vp] * 7 + [_vp] * 7),
    ("ork_b200_i8_mm_layer_async", _i, [_vp, _vp] + [_vp] * 7 + [_vp] * 7 + [_vp]),
    ("ork_b200_i8_mm_layers_async", _i, [_vp, _vp, _i, _vp, _vp, _vp, _vp]),
    ("ork_b200_rmsnorm_q8_async", _i, [_vp, _vp, _vp, _i, _vp, _vp]),
    ("ork_b200_argmax_scaled_async", _i, [_vp, _vp, _vp, _i, _vp]),
    ("ork_b200_rows_q8_async", _i, [_vp, _vp, _vp, _i, _i, _i, _vp, _vp]),
    ("ork_b200_rows_swiglu_q8_async", _i, [_vp, _vp, _vp, _i, _i, _vp, _vp, _vp]),
    ("ork_b200_rows_dequant_async", _i, [_vp, _vp, _i, _i, _vp, _vp, _vp, _vp]),
    ("ork_b200_rows_qk_rope_async", _i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _i, _f, _vp, _vp, _vp, _i]),
    ("ork_b200_pack_check", _i, [_vp, _sz, _i, _i, _i]),
    ("ork_b200_pack_capid", C.c_uint32, []),
    ("ork_b200_sync", _i, [_vp]),
    ("ork_b200_stream", _vp, [_vp]),
    ("ork_b200_set_stream", _i, [_vp, _vp]),
    ("ork_b200_device", _i, [_vp]),
    ("ork_b200_set_pdl", _i, [_vp, _i]),
    ("ork_b200_launches", C.c_uint64, [_vp]),
    ("ork_b200_weight_ptr", _vp, [_vp]),
    ("ork_b200_weight_read", _sz, [_vp, _vp, _sz]),
    ("ork_b200_route", _i, [_vp, _i]),
    ("ork_b200_force_route", _i, [_vp, _i]),
    ("ork_b200_tc_choice", _i, [_i, _i, _i, _i, _vp]),
    ("ork_b200_gemv_choice", _i, [_i, _i, _i, _i, _vp]),
    ("ork_b200_reload_tuning", _i, [_vp]),
    ("ork_b200_staging_bytes", _sz, [_vp]),
    ("ork_i4_mm_run_stream", _i, [_vp, _i, _vp]),
    ("ork_mm_run_async", _vp, [_vp, _vp, _i, _vp, _vp]),
    ("ork_i8_mm_run_async", _vp, [_vp, _vp, _i, _vp, _vp]),
    ("ork_i4_mm_run_async", _vp, [_vp, _vp, _i, _vp, _vp]),
    ("ork_i8_mm_run_chain_async", _vp, [_vp, _i, _vp]),
    ("ork_i4_mm_run_chain_async", _vp, [_vp, _i, _vp]),
    ("ork_i8_mm_run_stream_async", _vp, [_vp, _i, _vp]),
    ("ork_i4_mm_run_stream_async", _vp, [_vp, _i, _vp]),
    ("ork_async_wait", _i, [_vp]),
    ("ork_npu_last_async_cpu", _i, [_vp]),
]


def lib():
    """The loaded libork_npu.so, with every prototype declared."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libork_npu.so not built ({LIB_PATH}); run `make -C ork-driver_b200`")
        L = C.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Context:
    """One ork_npu context on the current CUDA device."""

    def __init__(self):
        self.L = lib()
        self.ctx = self.L.ork_npu_init()
        if not self.ctx:
            raise RuntimeError("ork_npu_init failed (no B200 visible?)")

    def close(self):
        if self.ctx:
            self.L.ork_npu_free(self.ctx)
            self.ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ---- pack -----------------------------------------------------------------------------------
    def i8_pack(self, B_kn):
        B_kn = np.ascontiguousarray(B_kn, np.int8)
        K, N = B_kn.shape
        return Weight(self, self.L.ork_i8_mm_pack(self.ctx, K, N, _p(B_kn)), K, N, "i8")

    def i8_pack_f32(self, f32_nk):
        f32_nk = np.ascontiguousarray(f32_nk, np.float32)
        N, K = f32_nk.shape
        bs = np.zeros(N, np.float32)
        w = Weight(self, self.L.ork_i8_mm_pack_f32(self.ctx, K, N, _p(f32_nk), _p(bs)), K, N, "i8")
        return w, bs

    def i4a8_pack(self, f32_nk, imatrix=None):
        f32_nk = np.ascontiguousarray(f32_nk, np.float32)
        N, K = f32_nk.shape
        bs = np.zeros(N, np.float32)
        if imatrix is None:
            h = self.L.ork_i4a8_mm_pack(self.ctx, K, N, _p(f32_nk), _p(bs))
        else:
            im = np.ascontiguousarray(imatrix, np.float32)
            h = self.L.ork_i4a8_mm_pack_im(self.ctx, K, N, _p(f32_nk), _p(im), _p(bs))
        return Weight(self, h, K, N, "i8"), bs

    def i4_pack(self, B_kn):
        B_kn = np.ascontiguousarray(B_kn, np.int8)
        K, N = B_kn.shape
        return Weight(self, self.L.ork_i4_mm_pack(self.ctx, K, N, _p(B_kn)), K, N, "i4")

    def f16_pack(self, B_kn):
        B_kn = np.ascontiguousarray(B_kn, np.float16)
        K, N = B_kn.shape
        return Weight(self, self.L.ork_f16_mm_pack(self.ctx, K, N, _p(B_kn)), K, N, "f16")

    def i4a8_load(self, blob, K, N):
        blob = np.ascontiguousarray(blob, np.uint8)
        return Weight(self, self.L.ork_i4a8_mm_load(self.ctx, K, N, _p(blob), blob.nbytes), K, N, "i8")

    def i4_pack_grouped(self, B_kn, G):
        B_kn = np.ascontiguousarray(B_kn, np.int8)
        K, N = B_kn.shape
        return Weight(self, self.L.ork_i4_mm_pack_grouped(self.ctx, K, N, _p(B_kn), G), K, N, "i4")

    def load(self, blob, K, N, kind):
        """ork_{i8,i4,f16}_mm_load of a stamped .orkpack blob."""
        blob = np.ascontiguousarray(blob, np.uint8)
        fn = {"i8": self.L.ork_i8_mm_load, "i4": self.L.ork_i4_mm_load, "f16": self.L.ork_f16_mm_load}[kind]
        return Weight(self, fn(self.ctx, K, N, _p(blob), blob.nbytes), K, N, kind)

    def i4a8_load_tiled(self, blob, K, N, G):
        blob = np.ascontiguousarray(blob, np.uint8)
        return Weight(self, self.L.ork_i4a8_mm_load_tiled(self.ctx, K, N, _p(blob), blob.nbytes, G), K, N, "i8")

    def dump_cpu(self, B_kn, kind):
        """ork_i8_w_dump_cpu / ork_i4_w_dump_cpu: the stamped blob, built on the host."""
        B_kn = np.ascontiguousarray(B_kn, np.int8)
        K, N = B_kn.shape
        fn = self.L.ork_i8_w_dump_cpu if kind == "i8" else self.L.ork_i4_w_dump_cpu
        need = fn(self.ctx, K, N, _p(B_kn), None, 0)
        out = np.zeros(need, np.uint8)
        assert need and fn(self.ctx, K, N, _p(B_kn), _p(out), need) == need
        return out

    def run_grouped(self, w, A, aS, bS):
        """ork_i4_mm_run_grouped / ork_i8_mm_run_grouped (by w's kind); returns (rc, C fp32)."""
        A = np.ascontiguousarray(A, np.int8)
        aS = np.ascontiguousarray(aS, np.float32)
        bS = np.ascontiguousarray(bS, np.float32)
        M = A.shape[0]
        Cm = np.zeros((M, w.N), np.float32)
        fn = self.L.ork_i4_mm_run_grouped if w.kind == "i4" else self.L.ork_i8_mm_run_grouped
        return fn(self.ctx, w.h, M, _p(A), _p(aS), _p(bS), _p(Cm)), Cm

    # ---- run (synchronous, host numpy buffers) ---------------------------------------------------
    def run(self, w, A, M=None):
        """C = A . B through the run function matching w's dtype; returns (rc, C)."""
        M = A.shape[0] if M is None else M
        if w.kind == "f16":
            A = np.ascontiguousarray(A, np.float16)
            Cm = np.zeros((M, w.N), np.float32)
            rc = self.L.ork_f16_mm_run(self.ctx, w.h, M, _p(A), _p(Cm))
        else:
            A = np.ascontiguousarray(A, np.int8)
            Cm = np.zeros((M, w.N), np.int32)
            fn = self.L.ork_i4_mm_run if w.kind == "i4" else self.L.ork_i8_mm_run
            rc = fn(self.ctx, w.h, M, _p(A), _p(Cm))
        return rc, Cm

    def launches(self):
        return int(self.L.ork_b200_launches(self.ctx))


class TaskI8(C.Structure):
    """ork_mm_task_i8 (include/ork_npu.h)."""
    _fields_ = [("w", C.c_void_p), ("M", C.c_int), ("A", C.c_void_p), ("C", C.c_void_p), ("cstride", C.c_int)]


class TaskI4(C.Structure):
    """ork_mm_task_i4 (include/ork_npu.h)."""
    _fields_ = [("w", C.c_void_p), ("M", C.c_int), ("A", C.c_void_p), ("C", C.c_void_p)]


class LayerDims(C.Structure):
    """struct ork_layer_dims (include/ork_npu.h)."""
    _fields_ = [(k, C.c_uint32) for k in ("D", "H", "Hkv", "dk", "dv", "Nff", "nkv", "pos")] + \
        [("attn_scale", C.c_double), ("rope_base", C.c_double)]


class LayerKV(C.Structure):
    """ork_b200_layer_kv (include/ork_b200.h)."""
    _fields_ = [("k_norm", C.c_void_p), ("append", C.c_int), ("hstride", C.c_int), ("dpos", C.c_void_p)]


class LayerW(C.Structure):
    """ork_b200_layer_w (include/ork_b200.h): one layer of ork_b200_i8_mm_layers_async."""
    _fields_ = [(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "attn_norm", "q_norm",
                                          "ffn_norm", "k_norm", "Kc", "Vc")]


class Weight:
    def __init__(self, ctx, handle, K, N, kind=None):
        self.ctx, self.h, self.K, self.N = ctx, handle, K, N
        self.kind = kind

    def __bool__(self):
        return bool(self.h)

    def free(self):
        if self.h:
            self.ctx.L.ork_mm_free(self.ctx.ctx, self.h)
            self.h = None

    def bscale(self):
        p = self.ctx.L.ork_w_bscale(self.h)
        if not p:
            return None
        return np.ctypeslib.as_array(p, shape=(self.N,)).copy()

    def quant_kind(self):
        return self.ctx.L.ork_w_quant_kind(self.h)

    def resident(self):
        """The weight's resident bytes (ork_b200_weight_read)."""
        need = self.ctx.L.ork_b200_weight_read(self.h, None, 0)
        out = np.zeros(need, np.uint8)
        assert self.ctx.L.ork_b200_weight_read(self.h, _p(out), need) == need
        return out

    def set_group(self, G):
        return self.ctx.L.ork_w_set_group(self.h, G)

    def pack_dump(self):
        """ork_w_dump: the stamped .orkpack entry of this weight."""
        need = self.ctx.L.ork_w_dump(self.h, None, 0)
        if need == 0:
            return None
        out = np.zeros(need, np.uint8)
        assert self.ctx.L.ork_w_dump(self.h, _p(out), need) == need
        return out

    def dump(self):
        need = self.ctx.L.ork_i4a8_w_dump(self.h, None, 0)
        if need == 0:
            return None
        out = np.zeros(need, np.uint8)
        got = self.ctx.L.ork_i4a8_w_dump(self.h, _p(out), need)
        assert got == need, (got, need)
        return out


def cpu_blob(f32_nk, imatrix=None, nf4=False, qerr=False):
    """ork_i4a8_pack_cpu_blob(_qerr): the library's host-only O4N1 writer (no device needed)."""
    L = lib()
    f32_nk = np.ascontiguousarray(f32_nk, np.float32)
    N, K = f32_nk.shape
    im = None if imatrix is None else np.ascontiguousarray(imatrix, np.float32)
    need = L.ork_i4a8_pack_cpu_blob(None, K, N, _p(f32_nk), _p(im), int(nf4), None, 0)
    out = np.zeros(need, np.uint8)
    q = C.c_float(-1.0)
    got = L.ork_i4a8_pack_cpu_blob_qerr(None, K, N, _p(f32_nk), _p(im), int(nf4), _p(out), need,
                                        C.byref(q) if qerr else None)
    assert got == need
    return (out, q.value) if qerr else out
