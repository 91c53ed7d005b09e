"""Host logic of the fused-gather peer group (ork-driver_b200/shard.py PeerGroup) on two gloo ranks on
CPU: every rank's symmetric buffers are exchanged as 64-byte handles, opened in rank order, and each
rank's peer table gets every rank's buffers in the same order with its own first column at
rank * ncols; close() releases the tables and mappings between two barriers. The library calls are
replaced by a recording fake (the IPC mapping itself needs GPUs; tests/test_gpu_peers.py runs it)."""
import ctypes as C
import os
import socket
import struct

import torch.multiprocessing as mp


class _FakeLib:
    def __init__(self, rank):
        self.rank, self.n, self.calls = rank, 0, []

    def ork_b200_sym_alloc(self, ctx, nbytes, h):
        self.n += 1
        ptr = (self.rank + 1) << 32 | self.n << 8
        C.memmove(h, struct.pack("<QQ", ptr, nbytes) + bytes(48), 64)
        self.calls.append(("alloc", ptr, nbytes))
        return ptr

    def ork_b200_sym_open(self, ctx, h):
        ptr, _ = struct.unpack("<QQ", bytes(h)[:16])
        self.calls.append(("open", ptr))
        return ptr | 1  # a mapping is a different address in this process

    def ork_b200_peers_create(self, ctx, world, rank, cps, fps, ldc, col0, ncols):
        self.calls.append(("create", world, rank, [cps[i] for i in range(world)], [fps[i] for i in range(world)],
                           ldc, col0, ncols))
        return 0x1000 + len(self.calls)

    def ork_b200_sync(self, ctx):
        self.calls.append(("sync",))
        return 0

    def ork_b200_peers_destroy(self, t):
        self.calls.append(("destroy", t))

    def ork_b200_sym_close(self, ctx, q):
        self.calls.append(("close", q))
        return 0

    def ork_b200_sym_free(self, ctx, p):
        self.calls.append(("free", p))
        return 0


class _FakeCtx:
    def __init__(self, rank):
        self.L, self.ctx = _FakeLib(rank), 7


def _worker(rank, world, port, q):
    import torch.distributed as dist

    import shard

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    ctx = _FakeCtx(rank)
    g = shard.PeerGroup(ctx, dist)
    t, own = g.table(4, 512, 256)
    g.close()
    q.put((rank, own, ctx.L.calls))
    dist.destroy_process_group()


def test_peer_group_exchange_on_gloo_ranks():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (own, calls)) for r, own, calls in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    allocs = {r: [c[1] for c in calls if c[0] == "alloc"] for r, (_, calls) in res.items()}
    for r, (own, calls) in res.items():
        create = [c for c in calls if c[0] == "create"][0]
        _, world, rank, cps, fps, ldc, col0, ncols = create
        assert (world, rank, ldc, col0, ncols) == (2, r, 512, 256 * r, 256)
        # rank order: own buffer as allocated, the peer's as opened (mapped) here
        assert cps[r] == allocs[r][0] and fps[r] == allocs[r][1]
        o = 1 - r
        assert cps[o] == allocs[o][0] | 1 and fps[o] == allocs[o][1] | 1
        assert own == allocs[r][0]
        kinds = [c[0] for c in calls]
        # teardown: sync, then tables, then mappings, then own buffers
        assert kinds.index("sync") < kinds.index("destroy") < kinds.index("close") < kinds.index("free")
