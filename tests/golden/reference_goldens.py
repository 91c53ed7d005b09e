"""Golden checksums hard-coded in the reference's own tests, and the recipes that rebuild their inputs.

The reference (ork-driver) validates its matmul path with fixed-seed LCG inputs and an FNV-1a 64 checksum
of the int32 / fp32 output. The constants below are copied from those tests (as data, with file:line), and
the generators rebuild the identical inputs by replaying the same LCG stream in the same order, so any
implementation of the matmul can be held to the reference's own known answers:

- examples/quant.c:72-81        7 int8 cases, frand() stream seeded 1, per-channel/per-row quantized.
- examples/test_matmul.c:611-612 2 fp16 cases, rnd() stream seeded 12345, weights reused over M={1,1,4,M}.
- examples/test_matmul.c:84-86   7 int8 "chain prefill" cases continuing that stream.
- examples/test_matmul.c:639-641 3 int8 cases at the end of main(), after every test in between has
                                 consumed its share of rnd() (skipped here by counting).

Every case yields (name, kind, M_list, K, N, A, B_kn, gold): A is [Mmax][K] (int8 or float16), B_kn is
[K][N] row-major, and gold is the FNV-1a 64 of the outputs of C = A[:m] . B for m in M_list, chained.
"""
import numpy as np

QUANT_C_GOLDENS = [  # examples/quant.c:72-75, 79-81
    (64, 2048, 512, 0x44e94f9c68925002),
    (16, 4096, 512, 0x70b268248f6790ab),
    (8, 6144, 256, 0xe0fb450b023ba66e),
    (1, 2048, 2048, 0x7313f30cba5d9aa7),
    (512, 2048, 2048, 0xc1bfa757281554ec),
    (128, 2048, 2048, 0xe4bd381d52fa0d8c),
    (64, 4096, 512, 0x8ee9e7f5d99078cd),
]

TEST_MATMUL_F16 = [  # examples/test_matmul.c:611-612 (check(): Ms = {1,1,4,M})
    (64, 2048, 256, 0x63da26feb5488edd),
    (256, 3584, 256, 0xd659053d19504e43),
]

TEST_MATMUL_CHAIN_PREFILL = [  # examples/test_matmul.c:79-80 shapes, :84-86 GOLD (one run each)
    (256, 18944, 3584, 0xb4d325e573e7037c),
    (256, 3584, 3584, 0x6084624fae4ea1cd),
    (256, 2048, 2048, 0x1fc8a45628241e4b),
    (128, 512, 1536, 0xa752ea8100ba7d54),
    (200, 1024, 2048, 0x21dc86bea3c1015f),
    (128, 2048, 16384, 0x5b98ab74d6e8947a),
    (96, 3584, 18944, 0x3fcd5ced1fed0f53),
]

TEST_MATMUL_CHECK_I8 = [  # examples/test_matmul.c:639-641 (check_i8(): Ms = {1,1,4,M})
    (512, 2048, 256, 0xda6b68f190453353),
    (256, 3584, 256, 0x454860dd91b46165),
    (256, 256, 32, 0xf23ebd149849d390),
]


def _rnd_draws_between_chain_prefill_and_check_i8():
    """rnd() values drawn by the tests main() runs between check_chain_prefill and check_i8
    (examples/test_matmul.c:621-634), each counted from its allocation loops."""
    n = 4 * (1 * 512 + 512 * 64)                                   # check_chain_i8 :127-137
    n += sum(m * 2048 + 2048 * 768 for m in (1, 8, 40, 96))        # check_chain_i8_bf :187-196
    n += sum(m * k + k * nn for k, nn, m in zip((2048, 512, 4096, 1536, 1024, 2048),
                                                (512, 256, 2048, 512, 512, 768),
                                                (64, 8, 1, 40, 128, 32)))  # check_stream_i8 :214-225
    n += 768 * 512 + 8 * 768 + 1536 * 256 + 33 * 1536              # check_chain_envelope :245-267
    n += 512 * 2048 + 8 * 2048                                     # check_pack_i8_f32 :285-286
    n += 512 * 2048 + 8 * 2048                                     # check_pack_i4a8 :313-314
    # check_pack_i4a8_imatrix :453-461: one draw per weight, two for the 5 outlier columns k%401==0
    # (k = 401, 802, 1203, 1604, 2005) of each of the 512 channels, then the 8x2048 activations.
    n += 512 * (2048 + 5) + 8 * 2048
    # check_pack_nf4_correct / check_nf4_accuracy_gate / check_dump_load_i4a8 draw from gauss() only.
    return n


def quant_c_case(lcg, M, K, N):
    """examples/quant.c:27-37: frand() A then B; per-channel / per-row absmax/127 scales; q8 rounding."""
    A = lcg.frand(M * K).reshape(M, K)
    B = lcg.frand(K * N).reshape(K, N)

    def q8(x):
        return np.clip(np.rint(x), -127, 127).astype(np.int8)

    mx = np.abs(B).max(axis=0)
    ws = np.where(mx > 0, mx / np.float32(127), np.float32(1)).astype(np.float32)
    Bq = q8((B / ws[None, :]).astype(np.float32))
    mxa = np.abs(A).max(axis=1)
    as_ = np.where(mxa > 0, mxa / np.float32(127), np.float32(1)).astype(np.float32)
    Aq = q8((A / as_[:, None]).astype(np.float32))
    return Aq, Bq


def cases(Lcg, which=("quant", "f16", "chain", "check_i8"), max_macs=None):
    """Yield golden cases in stream order. `Lcg` is the generator class of tests/oracle_ffi.py.
    max_macs skips (but still consumes the stream of) cases whose M*K*N exceeds it."""
    if "quant" in which:
        g = Lcg(1)
        for M, K, N, gold in QUANT_C_GOLDENS:
            Aq, Bq = quant_c_case(g, M, K, N)
            if max_macs is None or M * K * N <= max_macs:
                yield (f"quant_c_{M}x{K}x{N}", "i8", [M], K, N, Aq, Bq, gold)
    if not ({"f16", "chain", "check_i8"} & set(which)):
        return
    g = Lcg(12345)
    for M, K, N, gold in TEST_MATMUL_F16:
        A = g.rnd_f16(M * K).reshape(M, K)
        B = g.rnd_f16(K * N).reshape(K, N)
        if "f16" in which and (max_macs is None or M * K * N <= max_macs):
            yield (f"test_matmul_f16_{M}x{K}x{N}", "f16", [1, 1, 4, M], K, N, A, B, gold)
    saved = None
    for i, (M, K, N, gold) in enumerate(TEST_MATMUL_CHAIN_PREFILL):
        if i == 5:
            saved = g.sd.value  # examples/test_matmul.c:89 -- restored after the loop (:113)
        if "chain" in which and (max_macs is None or M * K * N <= max_macs):
            A = g.rnd_i8(M * K).reshape(M, K)
            B = g.rnd_i8(K * N).reshape(K, N)
            yield (f"test_matmul_chain_{M}x{K}x{N}", "i8", [M], K, N, A, B, gold)
        else:
            g.skip(M * K + K * N)
    g = Lcg(saved)
    g.skip(_rnd_draws_between_chain_prefill_and_check_i8())
    for M, K, N, gold in TEST_MATMUL_CHECK_I8:
        A = g.rnd_i8(M * K).reshape(M, K)
        B = g.rnd_i8(K * N).reshape(K, N)
        if "check_i8" in which and (max_macs is None or M * K * N <= max_macs):
            yield (f"test_matmul_check_i8_{M}x{K}x{N}", "i8", [1, 1, 4, M], K, N, A, B, gold)
