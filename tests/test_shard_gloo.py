"""Column-sharded matmul across ranks, on CPU (gloo, world_size 2).

Each rank quantizes only its channel range of the weight (NF4 + imatrix, exactly as the library's pack
does per channel), computes its C shard with the oracle as the local product, and the shards are
all-gathered and reassembled by ork-driver_b200/shard.py. The result must equal the unsharded oracle
product bit for bit, and each rank's O4N1 payload must equal the matching rows of the unsharded blob
(per-channel quantization makes the shards exact slices).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import shard

K, N = 256, 128


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights():
    from make_fixtures import seeded_imatrix, seeded_weights

    return seeded_weights(314, N, K), seeded_imatrix(314, K)


def _rank_main(rank, world, port, Ms, q):
    try:
        import torch.distributed as dist

        import oracle_ffi as of

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        f32, im = _weights()
        mine = shard.shard_rows_nk(f32, rank, world)
        blob = of.i4a8_blob(mine, im, nf4=True)
        codes, _, _ = of.i4a8_blob_codes(blob, K, mine.shape[0])
        full_blob = of.i4a8_blob(f32, im, nf4=True)
        n0, n1 = shard.shard_range(N, rank, world)
        nib = full_blob[20 + 4 * N:].reshape(N, K // 2)
        same_payload = np.array_equal(blob[20 + 4 * (n1 - n0):].reshape(n1 - n0, K // 2), nib[n0:n1])
        full_codes, _, _ = of.i4a8_blob_codes(full_blob, K, N)
        results = []
        for M in Ms:
            A = np.random.default_rng(M).integers(-128, 128, size=(M, K), dtype=np.int8)
            local = torch.from_numpy(of.gemm_i32(A, codes))
            C = shard.gather_columns(local, dist).numpy()
            results.append(bool(np.array_equal(C, of.gemm_i32(A, full_codes))))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, same_payload, results))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, None, repr(e)))


@pytest.mark.parametrize("world", [2])
def test_column_shard_gather_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    Ms = [1, 3, 8]
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, Ms, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same_payload, results in out:
        assert same_payload is not None, results
        assert same_payload, f"rank {rank}: shard blob is not a slice of the full blob"
        assert all(results), (rank, results)


def test_shard_range_rules():
    assert shard.shard_range(8192, 3, 8) == (3072, 4096)
    assert shard.shard_range(10240, 7, 8) == (8960, 10240)
    assert shard.shard_range(128256, 0, 8) == (0, 16032)
    with pytest.raises(ValueError):
        shard.shard_range(96, 0, 2)  # 48-channel shards are not a multiple of 32
    with pytest.raises(ValueError):
        shard.shard_range(1000, 0, 3)
    with pytest.raises(ValueError):
        shard.shard_range(128, 0, 2, align=128)  # W4A4 needs 64-channel shards at least


def test_gather_is_identity_for_one_rank():
    class One:
        @staticmethod
        def get_world_size(group=None):
            return 1

    x = torch.arange(12, dtype=torch.int32).reshape(3, 4)
    assert shard.gather_columns(x, One()) is x
