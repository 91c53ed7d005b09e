"""The benchmark's algorithmic byte and op counts (the numerators of every roofline fraction it reports),
pinned to the per-call formulas of the measurement plan: weight + A + C bytes per run (int8:
K*N + M*K + 4*M*N; the int32 C is part of the traffic), 2*M*K*N ops, and the grouped run's scale tables."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)  # module level needs no GPU: torch and the library load inside the workloads
    return mod


@pytest.mark.parametrize("K,N,M,want", [
    (2048, 6144, 1, 12_609_536),     # 12.61 MB: 1.92 us at 6555 GB/s
    (2048, 6144, 512, 26_214_400),   # 26.21 MB
    (6144, 2048, 512, 19_922_944),   # 19.92 MB: the dominant sweep kernel's bytes per launch
    (2048, 2048, 8, 4_276_224),
])
def test_w8a8_bytes_per_run(bench, K, N, M, want):
    assert bench.alg_bytes(K, N, M) == want


def test_sweep_step_totals(bench):
    assert len(bench.CONFIGS) == 12
    assert bench.STEP_BYTES == sum(K * N + M * K + 4 * M * N for K, N, M in bench.CONFIGS) == 150_669_312
    assert bench.STEP_OPS == sum(2 * M * K * N for K, N, M in bench.CONFIGS) == 38_109_446_144


def test_grouped_bytes(bench):
    # int4 weight + fp32 bScale[K/G][N] + int8 A + fp32 aScale[M][K/G] + fp32 C
    K, N, G, M = 2048, 2048, 128, 4
    assert bench.grouped_bytes(K, N, G, M) == K * N // 2 + (K // G) * N * 4 + M * K + M * (K // G) * 4 + 4 * M * N


def test_peaks_source(bench):
    hbm, bf16, src = bench.peaks()
    assert src in ("measured", "fallback") and hbm > 1000 and bf16 > 100
    if src == "fallback":
        assert (hbm, bf16) == (6650.0, 1590.0)
