"""Generate tests/golden/reference_fixtures.json from the reference's own compiled CPU code.

Runs ork-driver's offline CPU path (oracle/_ref/libork_ref.so, built by `make -C oracle ref` from the
reference sources) on small seeded inputs and records what it produced: O4N1 blob hashes and qerr of
ork_i4a8_pack_cpu_blob_qerr for every quantizer mode, the per-channel int8 scales of orki_chan_scales_f32,
the W4A4 int32 result checksum of ork_i4_mm_pack + ork_i4_mm_run on an offline context, and the fp32
results of the grouped-scale path (ork_i4_mm_pack_grouped + ork_i4_mm_run_grouped, orki_cpu_gemm_grouped). The fixture
pins the restated oracle (oracle/ork_oracle.c) where the reference tree is absent (the GPU box).

    python tests/golden/make_fixtures.py            # rewrites reference_fixtures.json
"""
import ctypes as C
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import oracle_ffi as of  # noqa: E402

OUT = os.path.join(HERE, "reference_fixtures.json")

# (name, K, N, nf4, imatrix?, sr?) -- shapes small enough for the CPU suite, modes covering every branch
I4A8_CASES = [
    ("uniform", 256, 64, 0, False, False),
    ("nf4", 256, 64, 1, False, False),
    ("uniform_im", 512, 64, 0, True, False),
    ("nf4_im", 512, 64, 1, True, False),
    ("uniform_sr", 256, 32, 0, False, True),
    ("nf4_sr", 256, 32, 1, False, True),
    ("uniform_im_sr", 256, 32, 0, True, True),
    ("nf4_im_sr", 256, 32, 1, True, True),
    ("uniform_big", 2048, 128, 0, True, False),
    ("nf4_big", 2048, 128, 1, True, False),
]


def seeded_weights(seed, N, K, scale=0.02):
    """[N][K] f32 ~ N(0, scale) with a few large outliers, so the imatrix clip search has work to do."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(scale)).astype(np.float32)
    idx = rng.integers(0, N * K, size=max(1, N * K // 500))
    w.reshape(-1)[idx] *= np.float32(8.0)
    return w


def seeded_imatrix(seed, K):
    rng = np.random.default_rng(seed + 1000)
    return (rng.random(K, dtype=np.float32) * np.float32(1.5) + np.float32(0.5)).astype(np.float32)


# grouped scales: (M, K, N, G, activation range) -- W4A4 (A int4) and W4A8 (A int8) over int4 weights
GROUPED_CASES = [(1, 1024, 128, 32, 8), (3, 2048, 192, 128, 8), (8, 1024, 64, 256, 128), (5, 4096, 128, 64, 128)]


def grouped_inputs(seed, M, K, N, G, a_range):
    """A [M][K] in [-a_range, a_range), int4 weights B [K][N], aScale [M][K/G], bScale [K/G][N]."""
    rng = np.random.default_rng(seed)
    A = rng.integers(-a_range, a_range, size=(M, K), dtype=np.int8)
    B = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
    aS = rng.uniform(1e-3, 3e-2, size=(M, K // G)).astype(np.float32)
    bS = rng.uniform(1e-3, 3e-2, size=(K // G, N)).astype(np.float32)
    return A, B, aS, bS


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def ref_blob(ref, f32, im, nf4, sr):
    N, K = f32.shape
    if sr:
        os.environ["ORK_SR"] = "1"
    else:
        os.environ.pop("ORK_SR", None)
    try:
        need = ref.ork_i4a8_pack_cpu_blob_qerr(None, K, N, of._p(f32), None, nf4, None, 0, None)
        out = np.zeros(need, np.uint8)
        q = C.c_float(0)
        got = ref.ork_i4a8_pack_cpu_blob_qerr(None, K, N, of._p(f32), None if im is None else of._p(im), nf4,
                                              of._p(out), need, C.byref(q))
        assert got == need
    finally:
        os.environ.pop("ORK_SR", None)
    return out, q.value


def main():
    ref = of.reference()
    if ref is None:
        sys.exit("oracle/_ref/libork_ref.so missing: run `make -C oracle ref` where the reference tree exists")
    fx = {"source": "ork-driver offline CPU path, oracle/_ref/libork_ref.so", "i4a8": {}, "chan_scales": {},
          "w4a4": {}}
    for i, (name, K, N, nf4, use_im, sr) in enumerate(I4A8_CASES):
        f32 = seeded_weights(100 + i, N, K)
        im = seeded_imatrix(100 + i, K) if use_im else None
        blob, qerr = ref_blob(ref, f32, im, nf4, sr)
        fx["i4a8"][name] = {"seed": 100 + i, "K": K, "N": N, "nf4": nf4, "imatrix": use_im, "sr": sr,
                            "blob_sha256": sha(blob), "blob_bytes": int(blob.size),
                            "qerr_f32_hex": np.float32(qerr).tobytes().hex()}
    # per-channel int8 scales (src/npu.c:854 orki_chan_scales_f32; exported, no static)
    ref.orki_chan_scales_f32.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
    for seed, (K, N) in ((7, (2048, 256)), (8, (64, 32))):
        f32 = seeded_weights(seed, N, K)
        inv = np.zeros(N, np.float32)
        bs = np.zeros(N, np.float32)
        ref.orki_chan_scales_f32(of._p(f32), K, N, of._p(inv), of._p(bs))
        fx["chan_scales"][f"{K}x{N}"] = {"seed": seed, "K": K, "N": N, "inv_sha256": sha(inv),
                                         "bscale_sha256": sha(bs)}
    # W4A4 offline: ork_i4_mm_pack keeps raw codes, ork_i4_mm_run = orki_cpu_gemm_i32
    ctx = ref.ork_npu_init_offline(b"rk3588")
    for seed, (M, K, N) in ((11, (8, 256, 128)), (12, (32, 512, 64))):
        rng = np.random.default_rng(seed)
        B = rng.integers(-8, 8, size=(K, N), dtype=np.int8)
        A = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
        w = ref.ork_i4_mm_pack(ctx, K, N, of._p(B))
        Cm = np.zeros((M, N), np.int32)
        assert ref.ork_i4_mm_run(ctx, w, M, of._p(A), of._p(Cm)) == 0
        ref.ork_w_free(w)
        fx["w4a4"][f"{M}x{K}x{N}"] = {"seed": seed, "M": M, "K": K, "N": N, "c_fnv64": of.fnv64(Cm)}
    # grouped scales: ork_i4_mm_pack_grouped + ork_i4_mm_run_grouped (W4A4, A int4) on the offline context,
    # and orki_cpu_gemm_grouped with int8 activations (the W4A8 grouped tier shares it)
    fx["grouped"] = {}
    for i, (M, K, N, G, ar) in enumerate(GROUPED_CASES):
        seed = 300 + i
        A, B, aS, bS = grouped_inputs(seed, M, K, N, G, ar)
        Cm = np.zeros((M, N), np.float32)
        if ar == 8:
            w = ref.ork_i4_mm_pack_grouped(ctx, K, N, of._p(B), G)
            assert w and ref.ork_i4_mm_run_grouped(ctx, w, M, of._p(A), of._p(aS), of._p(bS), of._p(Cm)) == 0
            ref.ork_w_free(w)
        else:
            assert ref.orki_cpu_gemm_grouped(M, K, N, G, of._p(A), of._p(B), of._p(aS), of._p(bS), of._p(Cm)) == 0
        fx["grouped"][f"{M}x{K}x{N}_G{G}_a{ar}"] = {"seed": seed, "M": M, "K": K, "N": N, "G": G, "a_range": ar,
                                                    "c_sha256": sha(Cm)}
    ref.ork_npu_free(ctx)
    with open(OUT, "w") as f:
        json.dump(fx, f, indent=1, sort_keys=True)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
