"""The library's host-side pack code against the oracle (CPU only): the O4N1 writer
ork_i4a8_pack_cpu_blob(_qerr) must emit byte-identical blobs to the restated reference for every quantizer
mode, and the same qerr as the reference's compiled code where that is available."""
import os

import numpy as np
import pytest

import oracle_ffi as of
import ork_b200
from make_fixtures import I4A8_CASES, seeded_imatrix, seeded_weights


@pytest.mark.parametrize("case", I4A8_CASES, ids=[c[0] for c in I4A8_CASES])
def test_library_cpu_blob_equals_oracle(env_clean, case):
    name, K, N, nf4, use_im, sr = case
    w = seeded_weights(200 + K + N, N, K)
    im = seeded_imatrix(200, K) if use_im else None
    if sr:
        env_clean.setenv("ORK_SR", "1")
    mine = ork_b200.cpu_blob(w, im, nf4=bool(nf4))
    assert np.array_equal(mine, of.i4a8_blob(w, im, nf4=bool(nf4), sr=bool(sr)))


@pytest.mark.skipif(of.reference() is None, reason="oracle/_ref not built")
@pytest.mark.parametrize("nf4", [0, 1])
@pytest.mark.parametrize("use_im", [False, True])
def test_library_qerr_equals_reference(env_clean, nf4, use_im):
    from make_fixtures import ref_blob

    K, N = 768, 64
    w = seeded_weights(5, N, K)
    im = seeded_imatrix(5, K) if use_im else None
    rblob, rq = ref_blob(of.reference(), w, im, nf4, False)
    blob, q = ork_b200.cpu_blob(w, im, nf4=bool(nf4), qerr=True)
    assert np.array_equal(blob, rblob)
    assert np.float32(q) == np.float32(rq)


def test_edge_values_quantize_like_oracle(env_clean):
    """All-zero channels, exact grid ties, clamped outliers, subnormals and +-1 normalised NF4 levels."""
    K, N = 64, 32
    w = np.zeros((N, K), np.float32)
    w[1, :] = np.linspace(-1, 1, K, dtype=np.float32)
    w[2, :] = 0.5  # uniform: 0.5/(0.5/7) = 7 exactly
    w[3, ::2], w[3, 1::2] = 3.5, -3.5
    w[4, :] = np.float32(1e-30)
    w[5, 0] = 1e6  # one huge outlier flattens the rest
    w[6, :] = np.arange(K, dtype=np.float32) * np.float32(0.5) - 16  # x.5 ties for rint
    w[7, :] = -0.0
    for nf4 in (False, True):
        assert np.array_equal(ork_b200.cpu_blob(w, None, nf4=nf4), of.i4a8_blob(w, None, nf4=nf4))
        im = np.ones(K, np.float32)
        assert np.array_equal(ork_b200.cpu_blob(w, im, nf4=nf4), of.i4a8_blob(w, im, nf4=nf4))


def test_blob_header_layout():
    K, N = 64, 32
    w = seeded_weights(1, N, K)
    blob = ork_b200.cpu_blob(w, None, nf4=True)
    hdr = np.frombuffer(blob[:20].tobytes(), np.uint32)
    assert hdr[0] == 0x4F344E31 and hdr[1] == 1 and hdr[2] == K and hdr[3] == N and hdr[4] == 1
    codes, bs, qk = of.i4a8_blob_codes(blob, K, N)
    assert qk == 1 and np.array_equal(bs, np.frombuffer(blob[20:20 + 4 * N].tobytes(), np.float32))
    assert set(np.unique(codes)) <= set(of.nf4_lut().tolist())


def test_oracle_refuses_malformed_blobs():
    K, N = 64, 32
    blob = ork_b200.cpu_blob(seeded_weights(2, N, K))
    assert of.i4a8_blob_codes(blob, K, N) is not None
    assert of.i4a8_blob_codes(blob[:-1], K, N) is None
    for off, val in ((0, 0), (4, 2), (8, 65), (12, 33), (16, 2)):
        bad = blob.copy()
        bad[off:off + 4] = np.frombuffer(np.uint32(val).tobytes(), np.uint8)
        assert of.i4a8_blob_codes(bad, K, N) is None, off
    assert of.i4a8_blob_codes(blob, K, N + 32) is None


def _nf4_boundary_rows(N=32, K=128, seed=9):
    """Rows of max |w| = 1 (so the normalised value is the weight itself) holding every NF4 level, its two
    float neighbours, every midpoint between adjacent levels and the midpoints' neighbours: the values on
    which a level search or the tie rule (t >= 0.5 goes up) could decide differently."""
    lv = np.array([-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
                   -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
                   0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
                   0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0], np.float32)
    mids = ((lv[:-1] + lv[1:]) / np.float32(2)).astype(np.float32)
    vals = []
    for x in np.concatenate([lv, mids]):
        vals += [x, np.nextafter(x, np.float32(-2)), np.nextafter(x, np.float32(2))]
    vals = np.clip(np.array(vals, np.float32), -1, 1)
    vals = np.concatenate([vals, np.array([-0.0], np.float32)])
    assert vals.size < K
    rng = np.random.default_rng(seed)
    w = np.zeros((N, K), np.float32)
    for n in range(N):
        row = np.concatenate([vals, np.zeros(K - vals.size, np.float32)])
        rng.shuffle(row)
        row[np.argmax(np.abs(row))] = np.float32(1.0 if n % 2 else -1.0)  # absmax exactly 1
        w[n] = row
    return w


def test_nf4_level_boundaries_quantize_like_oracle(env_clean):
    w = _nf4_boundary_rows()
    K = w.shape[1]
    for im in (None, np.ones(K, np.float32), seeded_imatrix(11, K)):
        assert np.array_equal(ork_b200.cpu_blob(w, im, nf4=True), of.i4a8_blob(w, im, nf4=True))


@pytest.mark.skipif(of.reference() is None, reason="oracle/_ref not built")
def test_nf4_level_boundaries_equal_reference(env_clean):
    """The same rows, and one with a NaN weight (its normalised value compares below no level: index 0),
    against ork-driver's own compiled quantizer, byte for byte."""
    from make_fixtures import ref_blob

    w = _nf4_boundary_rows()
    w[5, 7] = np.float32("nan")
    K = w.shape[1]
    for im in (None, seeded_imatrix(12, K)):
        rblob, _ = ref_blob(of.reference(), w, im, 1, False)
        assert np.array_equal(ork_b200.cpu_blob(w, im, nf4=True), rblob)
