"""N-column sharding of one GEMM across the GPUs of a box (one process per GPU).

The reference has no multi-GPU code; BASELINE's config-5 shape
(M=16384, N=65536, K=8192) is split column-wise: rank g holds all of A (M x K,
replicated), the contiguous row slab B[n0:n1, :] of B (N x K, K contiguous) and
writes its own slab C_g = A . B[n0:n1]^T (M x (n1-n0), contiguous). The compute
needs no exchange. An optional all-gather of the C slabs over NVLink (NCCL) gives
[G][M][N/G]; `relayout_gathered` turns that into row-major M x N. `GatheredC` is the
fused alternative: the GEMM epilogue itself stores every C tile into a symmetric
M x N buffer on every GPU (one multimem store through the NVSwitch per 16 bytes, or
peer stores where the node has no NVLink multicast), so the gather overlaps the
remaining tiles' math and needs no re-layout.

Host logic only (plain integer arithmetic plus torch.distributed calls); the GEMM
itself is b200_gemm on each rank's device.
"""
from __future__ import annotations


def shard_columns(n: int, world: int, rank: int, align: int = 16) -> tuple[int, int]:
    """Contiguous [n0, n1) of the N columns owned by `rank`.

    Boundaries are multiples of `align` (16 keeps every C slab's row length a
    16-byte multiple for 8-bit to 32-bit outputs) except the last, which ends at n.
    Ranks get near-equal shares; trailing ranks may get an empty range when n is
    small.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if n < 0 or align < 1:
        raise ValueError("n must be >= 0 and align >= 1")
    units = -(-n // align)  # ceil
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    return min(n, u0 * align), min(n, u1 * align)


def shard_sizes(n: int, world: int, align: int = 16) -> list[int]:
    return [b - a for a, b in (shard_columns(n, world, r, align) for r in range(world))]


def relayout_gathered(gathered, sizes=None):
    """[G][M][Ng] (all-gather of equal C slabs) -> row-major [M][G*Ng].

    With unequal slabs pass `sizes` and a list of [M][Ng_g] tensors instead.
    """
    import torch

    if sizes is None:
        g, m, ng = gathered.shape
        return gathered.permute(1, 0, 2).reshape(m, g * ng).contiguous()
    return torch.cat(list(gathered), dim=1).contiguous()


def gemm_shard(b200, a, b_full_or_slab, c_slab, rank: int, world: int, slab_given: bool = True,
               **kw):
    """Compute this rank's C slab. With slab_given=False, slice B's row slab here."""
    if slab_given:
        b_slab = b_full_or_slab
    else:
        n0, n1 = shard_columns(b_full_or_slab.shape[0], world, rank)
        b_slab = b_full_or_slab[n0:n1]
    if b_slab.shape[0] == 0:
        return c_slab
    return b200.gemm(a, b_slab, c_slab, **kw)


class GatheredC:
    """Row-major M x N output allocated in symmetric memory on every rank of `group`,
    written by b200_gemm_allgather from every rank's C slab.

    The buffer comes from torch.distributed._symmetric_memory (PyTorch is the plumbing
    here: it allocates the peer-mapped memory, binds it to an NVLink multicast object
    when the node supports one and exchanges the handles over the process group).
    """

    def __init__(self, m: int, n: int, dtype, device, group=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.m, self.n = m, n
        self.buf = symm_mem.empty((m, n), dtype=dtype, device=device)
        self.handle = symm_mem.rendezvous(self.buf, self.group)
        # 0 when the node has no NVLink multicast (NVLS) for this buffer
        self.multicast = int(self.handle.multicast_ptr) != 0
        # device array of every rank's base address (GATHER_PEERS)
        self.peer_bases = torch.tensor([int(p) for p in self.handle.buffer_ptrs], dtype=torch.int64,
                                       device=device)

    def slab(self, n_total: int | None = None) -> tuple[int, int]:
        return shard_columns(n_total or self.n, self.world, self.rank)

    def gemm(self, b200, a, b_slab, c_slab, *, force_peers: bool = False, stream=None, **kw):
        """This rank's C slab = A . B_slab^T, stored locally into `c_slab` and into the
        gathered buffer of every rank at this rank's columns. Queued on `stream`."""
        n0, n1 = self.slab()
        if n1 - n0 != b_slab.shape[0]:
            raise ValueError("B slab does not match this rank's columns")
        if n1 == n0:
            return c_slab
        if self.multicast and not force_peers:
            dst, mode, npeers = self.handle.multicast_ptr, b200.GATHER_MULTICAST, 0
        else:
            dst, mode, npeers = self.peer_bases.data_ptr(), b200.GATHER_PEERS, self.world
        return b200.gemm_allgather(a, b_slab, c_slab, dst, mode, npeers, self.n, n0, stream=stream,
                                   **kw)

    def sync(self):
        """Every rank's gathered stores are complete and visible (a barrier on the
        symmetric memory's signal pads, queued on the current stream)."""
        self.handle.barrier(channel=0)


def all_gather_columns(c_slab, world: int, group=None):
    """All-gather equal-size C slabs from every rank and re-lay them out as M x N."""
    import torch
    import torch.distributed as dist

    m, ng = c_slab.shape
    gathered = torch.empty((world, m, ng), dtype=c_slab.dtype, device=c_slab.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, c_slab.contiguous(), group=group)
    else:  # gloo (CPU tests) has only the list form
        dist.all_gather(list(gathered.unbind(0)), c_slab.contiguous(), group=group)
    return relayout_gathered(gathered)
