"""Column sharding of resident weights across the GPUs of one node (the 70B-shape configuration).

Output channels are independent in every format of this library -- each channel has its own scale and
its own K codes (ork-driver src/npu/i4/pack.c:63-80) -- so a weight B[K,N] splits by channel ranges with
no change to any value: rank g packs channels [g*N/G, (g+1)*N/G) (a contiguous row block of the n-major
f32 source) and produces C[:, its range]. The reference splits the same way across its NPU cores
(src/npu.c:1356-1398). One collective per sharded matmul reassembles C: an all-gather of the int32
shards over NCCL (NVLink / NVSwitch), then a channel-order view. Shard widths must keep the pack's
alignment (N/G a multiple of 32, of 64 for W4A4).

The module keeps the collective separate from the local matmul so the host-side logic (slicing, the
gather and reassembly order) is testable on CPU ranks with any local product.
"""
import numpy as np


def shard_range(N, rank, world, align=32):
    """Channel range [n0, n1) of `rank` for an N-channel weight split over `world` ranks."""
    if N % world or (N // world) % align:
        raise ValueError(f"N={N} does not split into {world} shards of a multiple of {align} channels")
    w = N // world
    return rank * w, (rank + 1) * w


def shard_rows_nk(f32_nk, rank, world, align=32):
    """This rank's rows of an n-major [N][K] f32 weight (what ork_i8_mm_pack_f32 / ork_i4a8_mm_pack take)."""
    n0, n1 = shard_range(f32_nk.shape[0], rank, world, align)
    return np.ascontiguousarray(f32_nk[n0:n1])


def shard_cols_kn(b_kn, rank, world, align=32):
    """This rank's columns of a row-major [K][N] weight (what ork_i8_mm_pack / ork_i4_mm_pack take)."""
    n0, n1 = shard_range(b_kn.shape[1], rank, world, align)
    return np.ascontiguousarray(b_kn[:, n0:n1])


def gather_columns(local, dist, group=None, out=None):
    """All-gather the [M][N/G] shards of all ranks and return C [M][N] in channel order.

    `local` is a torch tensor (int32 or float32) on the rank's device (CUDA with NCCL, CPU with gloo).
    The collective gathers [G][M][N/G]; for M = 1 that is already [N], otherwise the rank axis moves next
    to the channel axis (one strided copy)."""
    import torch

    world = dist.get_world_size(group)
    M, w = local.shape
    if world == 1:
        return local
    local = local.contiguous()
    if dist.get_backend(group) == "nccl":
        stacked = torch.empty((world, M, w), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(stacked, local, group=group)
    else:
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local, group=group)
        stacked = torch.stack(parts)
    if M == 1:
        full = stacked.view(1, world * w)
    else:
        full = stacked.permute(1, 0, 2).reshape(M, world * w)
    if out is not None:
        out.copy_(full)
        return out
    return full


class ShardedLinear:
    """One column-sharded resident weight on this rank, run through the library's async device-pointer
    call, followed by the all-gather of C."""

    def __init__(self, ctx, weight, N, rank, world):
        self.ctx, self.w, self.N, self.rank, self.world = ctx, weight, N, rank, world
        self.n0, self.n1 = shard_range(N, rank, world)

    def forward(self, A_dev, C_local, dist, C_full=None):
        L = self.ctx.L
        M = A_dev.shape[0]
        fn = L.ork_b200_i4_mm_run_async if self.w.kind == "i4" else L.ork_b200_i8_mm_run_async
        if fn(self.ctx.ctx, self.w.h, M, A_dev.data_ptr(), C_local.data_ptr()) != 0:
            raise RuntimeError("sharded matmul launch failed")
        return gather_columns(C_local, dist, out=C_full)


class PeerGroup:
    """Fused-gather runs over NVLink peer memory (ork_b200_peers_*, include/ork_b200.h): symmetric buffers
    allocated by the library on every rank, their CUDA IPC handles exchanged with `dist`
    (all_gather_object, any backend), each peer's buffer mapped here. `table(M, N, ncols)` returns a peer
    table for a weight whose N output channels are split into equal shards of `ncols` (this rank's
    first column = rank * ncols) and the device address of this rank's full C [M][N] int32."""

    HANDLE = 64

    def __init__(self, ctx, dist, group=None):
        self.ctx, self.dist, self.group = ctx, dist, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.own, self.opened, self.tables = [], [], []

    def _symmetric(self, nbytes):
        import ctypes as C

        L = self.ctx.L
        h = (C.c_uint8 * self.HANDLE)()
        p = L.ork_b200_sym_alloc(self.ctx.ctx, nbytes, h)
        if not p:
            raise RuntimeError("ork_b200_sym_alloc failed")
        self.own.append(p)
        handles = [bytes(h)]
        if self.world > 1:
            handles = [None] * self.world
            self.dist.all_gather_object(handles, bytes(h), group=self.group)
        ptrs = []
        for r in range(self.world):
            if r == self.rank:
                ptrs.append(p)
                continue
            q = L.ork_b200_sym_open(self.ctx.ctx, (C.c_uint8 * self.HANDLE).from_buffer_copy(handles[r]))
            if not q:
                raise RuntimeError(f"ork_b200_sym_open failed for rank {r}")
            self.opened.append(q)
            ptrs.append(q)
        return ptrs

    def table(self, M, N, ncols, land=False):
        """land=True also attaches landing buffers (M x N tagged 8-byte words per rank), so run + gather
        calls of up to M rows take the tagged-word gather (ork_b200_peers_land)."""
        import ctypes as C

        if ncols * self.world != N:
            raise ValueError("shards must tile N exactly")
        cps = self._symmetric(M * N * 4)
        fps = self._symmetric(4 * 8)
        arr = C.c_void_p * self.world
        t = self.ctx.L.ork_b200_peers_create(self.ctx.ctx, self.world, self.rank, arr(*cps), arr(*fps), N,
                                             self.rank * ncols, ncols)
        if not t:
            raise RuntimeError("ork_b200_peers_create failed")
        self.tables.append(t)
        if land:
            lps = self._symmetric(M * N * 8)
            if self.ctx.L.ork_b200_peers_land(t, arr(*lps), M) != 0:
                raise RuntimeError("ork_b200_peers_land failed")
        return t, cps[self.rank]

    def close(self):
        L = self.ctx.L
        L.ork_b200_sync(self.ctx.ctx)
        if self.world > 1:
            self.dist.barrier(group=self.group)  # no rank unmaps while a peer may still store into it
        for t in self.tables:
            L.ork_b200_peers_destroy(t)
        for q in self.opened:
            L.ork_b200_sym_close(self.ctx.ctx, q)
        if self.world > 1:
            self.dist.barrier(group=self.group)
        for p in self.own:
            L.ork_b200_sym_free(self.ctx.ctx, p)
        self.own, self.opened, self.tables = [], [], []
