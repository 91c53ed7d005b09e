"""Parity on every BASELINE config, through the default router (needs a B200).

Each test packs its weight exactly as the config says, runs every M of the config through the public
synchronous call with the router's own kernel and tile choice (no forced route, no tuning variables),
and compares C with the CPU oracle: bit-exact int32 for w8a8 / w4a8 (uniform and NF4) / W4A4, fp32 within
max|err| <= 1e-3 * sqrt(K) * max|A| * max|B| for fp16 -- the reference's own per-shape gates
(examples/quant.c:72-81, examples/test_matmul.c:611-641) applied to the benchmark's shapes.

configs[4] (70B-shape NF4 linears) runs at its real sizes, at full width and at the column-shard width
each rank of a 2-, 4- and 8-GPU run holds: the shard's result must be the matching column block of the
unsharded oracle result. Its weights are O4N1 blobs of random NF4 codes and scales (the quantizer that
normally writes them is pinned byte for byte elsewhere), so the kernels see every code value at these
shapes without a 0.5 G-weight host quantization per case.
"""
import numpy as np
import pytest

import oracle_ffi as of
import ork_b200
from make_fixtures import seeded_imatrix, seeded_weights

pytestmark = pytest.mark.gpu

W8A8_SHAPES = [(2048, 2048), (2048, 6144), (6144, 2048)]
W8A8_MS = [1, 8, 128, 512]
W4_SHAPES = [(6144, 2048), (2048, 12288)]
W4_MS = [1, 32, 256]
L70 = [("qkv", 8192, 10240), ("o", 8192, 8192), ("gate_up", 8192, 57344), ("down", 28672, 8192),
       ("lm_head", 8192, 128256)]
L70_MS = [1, 8, 256]


@pytest.fixture(autouse=True)
def default_router(ctx):
    L = ork_b200.lib()
    assert L.ork_b200_force_route(ctx.ctx, -1) == 0
    assert L.ork_b200_reload_tuning(ctx.ctx) == 0
    yield


def f16_tol(A, B):
    K = A.shape[1]
    return 1e-3 * np.sqrt(K) * float(np.abs(A.astype(np.float32)).max()) * float(np.abs(B.astype(np.float32)).max())


def test_configs0_fp16(ctx):
    """ork_f16_mm_pack / ork_f16_mm_run, K=2048, N=6144, M in {1, 64}, A ~ U(-1,1),
    B ~ N(0,0.02)."""
    K, N = 2048, 6144
    rng = np.random.default_rng(2048_6144)
    B = (rng.standard_normal((K, N)) * 0.02).astype(np.float16)
    w = ctx.f16_pack(B)
    try:
        for M in (1, 64):
            A = rng.uniform(-1, 1, size=(M, K)).astype(np.float16)
            rc, Cm = ctx.run(w, A)
            assert rc == 0
            assert np.abs(Cm - of.gemm_f16(A, B)).max() <= f16_tol(A, B), M
    finally:
        w.free()


@pytest.mark.parametrize("K,N", W8A8_SHAPES)
def test_configs1_w8a8(ctx, K, N):
    """ork_i8_mm_pack_f32 of B f32 [N][K] ~ N(0,0.02), A int8 ~ U[-127,127], every M of the
    sweep; codes and scales as the oracle's quantizer, C bit-exact."""
    f32 = seeded_weights(31 * K + N, N, K)
    w, bs = ctx.i8_pack_f32(f32)
    codes, obs = of.i8_quant_f32(f32)
    assert np.array_equal(bs, obs)
    B = np.ascontiguousarray(codes.T)
    rng = np.random.default_rng(K + 3 * N)
    try:
        for M in W8A8_MS:
            A = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
            rc, Cm = ctx.run(w, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, B)), M
    finally:
        w.free()


@pytest.mark.parametrize("nf4", [False, True])
@pytest.mark.parametrize("K,N", W4_SHAPES)
def test_configs2_w4a8(ctx, env_clean, K, N, nf4):
    """configs[2] w4a8: ork_i4a8_mm_pack_im with imatrix ~ U(0.5,2), uniform grid and (ORK_NF4) the NF4
    codebook; the blob equals the oracle's, C bit-exact at every M."""
    if nf4:
        env_clean.setenv("ORK_NF4", "1")
    f32 = seeded_weights(K * 5 + N + nf4, N, K)
    im = seeded_imatrix(K + 9, K)
    w, _ = ctx.i4a8_pack(f32, im)
    blob = w.dump()
    assert np.array_equal(blob, of.i4a8_blob(f32, im, nf4=nf4))
    codes, _, qk = of.i4a8_blob_codes(blob, K, N)
    assert qk == int(nf4)
    rng = np.random.default_rng(K * 11 + N + nf4)
    try:
        for M in W4_MS:
            A = rng.integers(-127, 128, size=(M, K), dtype=np.int8)
            rc, Cm = ctx.run(w, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, codes)), M
    finally:
        w.free()


@pytest.mark.parametrize("K,N", W4_SHAPES)
def test_configs2_w4a4(ctx, K, N):
    """configs[2] W4A4: ork_i4_mm_pack of int4 B, A int4 ~ U[-7,7] in int8, ork_i4_mm_run, C bit-exact."""
    rng = np.random.default_rng(K * 13 + N)
    B = rng.integers(-7, 8, size=(K, N), dtype=np.int8)
    w = ctx.i4_pack(B)
    try:
        for M in W4_MS:
            A = rng.integers(-7, 8, size=(M, K), dtype=np.int8)
            rc, Cm = ctx.run(w, A)
            assert rc == 0 and np.array_equal(Cm, of.gemm_i32(A, B)), M
    finally:
        w.free()


def o4n1(nib_nk2, bscale, K, N, kind=1):
    """An O4N1 blob (src/npu/internal.h:584,597): header, bscale[N] f32, nibbles [N][K/2]."""
    hdr = np.array([0x4F344E31, 1, K, N, kind], dtype=np.uint32).view(np.uint8)
    return np.concatenate([hdr, bscale.astype(np.float32).view(np.uint8), nib_nk2.reshape(-1)])


@pytest.mark.parametrize("name,K,N", L70, ids=[x[0] for x in L70])
def test_configs4_nf4_linears_full_and_sharded(ctx, name, K, N):
    """each 70B-shape linear as an NF4 weight at full width and as the column shard of rank 0
    and of the last rank for 2, 4 and 8 GPUs (shard.shard_range), M in {1, 8, 256}; every result bit-exact
    against the unsharded oracle's matching columns."""
    import shard

    rng = np.random.default_rng(K * 7 + N)
    nib = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    bs = rng.uniform(1e-4, 1e-3, size=N).astype(np.float32)
    codes, _, qk = of.i4a8_blob_codes(o4n1(nib, bs, K, N), K, N)
    assert qk == 1
    As = {M: rng.integers(-127, 128, size=(M, K), dtype=np.int8) for M in L70_MS}
    refs = {M: of.gemm_i32(A, codes) for M, A in As.items()}
    del codes
    parts = [(0, N)]
    for world in (2, 4, 8):
        for rank in (0, world - 1):
            parts.append(shard.shard_range(N, rank, world))
    for n0, n1 in dict.fromkeys(parts):
        w = ctx.i4a8_load(o4n1(np.ascontiguousarray(nib[n0:n1]), bs[n0:n1], K, n1 - n0), K, n1 - n0)
        assert w
        try:
            for M, A in As.items():
                rc, Cm = ctx.run(w, A)
                assert rc == 0 and np.array_equal(Cm, refs[M][:, n0:n1]), (n0, n1, M)
        finally:
            w.free()
