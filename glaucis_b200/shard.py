"""Multi-GPU partitioning of the two workloads, one process per GPU.

Grouped matmul (by expert group): the rows of the ragged group list are cut
into `world` contiguous ranges at 128-row boundaries, balanced by row count; a
cut may fall inside a group, whose expert weights then live on both ranks.
Rank r multiplies its rows by its experts' weights (a smaller ragged problem
with its own group sizes) and the output rows are assembled on every rank
either by one NCCL all-gather of equal (padded) slabs after the matmul
(`all_gather_rows`), or overlapped with it: the rows are computed in chunks
straight into IPC-shared output buffers (`PeerBuffers`) and every finished
chunk, a contiguous block of rows, is copied into each peer's buffer by the
copy engines over NVLink while the next chunk is computed, or inside the
matmul itself (`gmm_fp8_fwd_gathered`): its epilogue TMA-stores every
finished slice of rows into every rank's buffer.  Each output
element is computed in the same K-block order as on one GPU, so the gathered
output equals the single-GPU one bit for bit.

Chunked GLA (by head): heads are cut into contiguous ranges; each rank runs
the forward on its heads (its own [B, T, H_r, K] tensors) and the outputs are
gathered head-major ([world, B, T, H_r, V]).

No reference counterpart (the reference evaluates on one TPU slice); the
partitioning follows the planned sharding of the grouped matmul by expert
group with an output all-gather and of GLA by batch x head.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import numpy as np
import torch

TILE = 128


@dataclass
class GmmShard:
    r0: int             # first global row of this rank
    r1: int             # one past its last row
    g0: int             # first group touching [r0, r1)
    g1: int             # one past the last group touching it
    sizes: np.ndarray   # int32 [g1 - g0]: this rank's rows of each of those groups

    @property
    def rows(self) -> int:
        return self.r1 - self.r0


def gmm_partition(group_sizes, world: int, tile: int = TILE) -> List[GmmShard]:
    """Contiguous row ranges, one per rank, cut at multiples of `tile` rows
    nearest to equal shares of the assigned rows (sum of group_sizes)."""
    sizes = np.asarray(group_sizes, dtype=np.int64)
    if (sizes < 0).any():
        raise ValueError("group sizes must be non-negative")
    off = np.concatenate([[0], np.cumsum(sizes)])
    total = int(off[-1])
    cuts = [0]
    for k in range(1, world):
        c = int(round(total * k / world / tile)) * tile
        cuts.append(min(max(c, cuts[-1]), total))
    cuts.append(total)
    shards = []
    for r in range(world):
        r0, r1 = cuts[r], cuts[r + 1]
        if r1 <= r0:
            shards.append(GmmShard(r0, r0, 0, 0, np.zeros(0, np.int32)))
            continue
        g0 = int(np.searchsorted(off, r0, side="right") - 1)
        g1 = int(np.searchsorted(off, r1, side="left"))
        loc = [max(0, min(int(off[g + 1]), r1) - max(int(off[g]), r0)) for g in range(g0, g1)]
        shards.append(GmmShard(r0, r1, g0, g1, np.asarray(loc, np.int32)))
    return shards


def gla_head_partition(H: int, world: int) -> List[range]:
    """Contiguous head ranges, sizes differing by at most one."""
    return [range(H * r // world, H * (r + 1) // world) for r in range(world)]


def all_gather_rows(local: torch.Tensor, counts: List[int], out: torch.Tensor) -> torch.Tensor:
    """Assembles `out` [sum(counts), ...] from every rank's `local`
    [counts[rank], ...] (rank order = row order).  Equal counts gather
    straight into `out`; unequal ones through slabs padded to the largest."""
    import torch.distributed as dist
    world = dist.get_world_size()
    width = max(counts)
    nccl = dist.get_backend() == "nccl"
    if all(c == width for c in counts) and nccl:
        dist.all_gather_into_tensor(out, local.contiguous())
        return out
    pad = local.new_zeros((width,) + tuple(local.shape[1:]))
    pad[: local.shape[0]] = local
    if nccl:
        slabs = local.new_empty((world * width,) + tuple(local.shape[1:]))
        dist.all_gather_into_tensor(slabs, pad)
        parts = list(slabs.split(width))
    else:
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad)
    r = 0
    for k, c in enumerate(counts):
        out[r:r + c] = parts[k][:c]
        r += c
    return out


def ring_order(items: list, rank: int) -> list:
    """`items` (one per rank) starting at this rank's and continuing round
    the ring: the order in which a rank's scatter epilogue stores every
    slice, so that at any moment the ranks store into different peers (their
    NVLink ingress spread evenly) rather than all into rank 0 first."""
    return list(items[rank:]) + list(items[:rank])


class _CudaArray:
    """A raw device allocation seen through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3, "strides": None}


def tensor_at(ptr: int, shape) -> torch.Tensor:
    """A bf16 tensor over device memory at `ptr` (own or peer-mapped), shape `shape`."""
    return torch.as_tensor(_CudaArray(ptr, shape, "<i2"), device="cuda").view(torch.bfloat16)


class PeerBuffers:
    """One [rows, N] bf16 buffer per rank, every rank's buffer mapped into
    every process (CUDA IPC over NVLink, unicast; no multicast object), for
    peer copies or gl_gmm_fp8_fwd_scatter.  `ptrs[r]` is rank r's buffer as seen from this
    process; `local` is this rank's buffer as a tensor.  Collective: every
    rank constructs and closes it together."""

    def __init__(self, rows: int, cols: int):
        import ctypes
        import torch.distributed as dist
        from . import _lib
        self._lib = _lib.load()
        rank, world = dist.get_rank(), dist.get_world_size()
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        rc = self._lib.gl_ipc_alloc(rows * cols * 2, ctypes.byref(ptr), handle)
        self._own = ptr.value if rc == 0 else None
        # every rank learns every rank's outcome, so that all of them raise
        # together (no rank is left waiting in a collective)
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle) if rc == 0 else None)
        if any(h is None for h in handles):
            if self._own:
                self._lib.gl_ipc_free(self._own)
            raise RuntimeError("peer buffer allocation failed on a rank")
        self.ptrs, self._opened = [], []
        opened_all = True
        for r, hb in enumerate(handles):
            if r == rank:
                self.ptrs.append(self._own)
                continue
            peer = ctypes.c_void_p()
            if self._lib.gl_ipc_open((ctypes.c_ubyte * 64).from_buffer_copy(hb), ctypes.byref(peer)) != 0:
                opened_all = False
                break
            self.ptrs.append(peer.value)
            self._opened.append(peer.value)
        flag = torch.tensor([1 if opened_all else 0], dtype=torch.int32, device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()) == 0:
            self.local = None
            self.close()
            raise RuntimeError("peer buffer mapping failed on a rank")
        self.local = tensor_at(self._own, (rows, cols))

    def close(self) -> None:
        """Unmaps the peers and frees this rank's buffer (after a barrier, so
        no rank still writes into it)."""
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier()  # no rank writes any more
        for p in self._opened:
            self._lib.gl_ipc_close(p)
        self._opened = []
        self.local = None
        dist.barrier()  # every rank has unmapped this rank's buffer
        self._lib.gl_ipc_free(self._own)
        self._own = None


def gmm_fp8_fwd_gathered(a_q: torch.Tensor, a_s: torch.Tensor, b_q: torch.Tensor, b_s: torch.Tensor,
                         me: GmmShard, peers: PeerBuffers,
                         group_sizes: torch.Tensor = None) -> torch.Tensor:
    """This rank's part of an expert-sharded grouped matmul, with the output
    assembled on every rank by the matmul itself: the rows of `me` (a_q / a_s
    are this rank's rows me.r0:me.r1, quantised 1x128; b_q / b_s the weights
    of groups me.g0:me.g1) are multiplied and each finished 32-row slice is
    TMA-stored from the epilogue into every rank's `peers` buffer at row
    me.r0 + m, over NVLink, while the next tile is computed
    (gl_gmm_fp8_fwd_scatter).  A stream-ordered all-reduce of one int then
    orders the readers, so when the current stream reaches it every rank's
    rows are in `peers.local`, which is returned ([sum of rows, N] bf16).
    The result IS the shared buffer: it stays valid until the next call,
    which overwrites it on every rank.  That call's kernels start only after
    a second stream-ordered all-reduce of one int that every rank enqueues
    before its kernel, so no rank stores into a peer's buffer while that
    peer's stream still has earlier work on it (reads of the previous result
    enqueued before the call).  Collective: every rank calls it, in the same
    order.  Each output element is computed in the single-GPU K-block order,
    so the assembled output equals a one-GPU gl_gmm_fp8_fwd bit for bit.
    `group_sizes` (int32, on the device) may hold me.sizes already, saving a
    host-to-device copy."""
    import torch.distributed as dist
    from . import ops
    # write-after-read order across calls: every rank's earlier stream work
    # on its buffer precedes this all-reduce, which precedes every store
    flag = torch.zeros(1, dtype=torch.int32, device=peers.local.device)
    dist.all_reduce(flag)
    if me.rows:
        if a_q.shape[0] != me.rows or b_q.shape[0] != me.g1 - me.g0:
            raise ValueError("a_q must hold this rank's rows and b_q its groups' weights")
        gs = group_sizes
        if gs is None:
            gs = torch.from_numpy(np.ascontiguousarray(me.sizes, np.int32)).to(a_q.device)
        ops.gmm_fp8_fwd_scatter(a_q, a_s, b_q, b_s, gs, ring_order(peers.ptrs, dist.get_rank()),
                                me.r0)
    dist.all_reduce(flag)
    return peers.local


def gla_fwd_gathered(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                     h0: torch.Tensor, scale: float, peers: PeerBuffers, width: int,
                     ht: torch.Tensor = None, exact_intra: bool = True) -> torch.Tensor:
    """This rank's heads of a head-sharded chunked-GLA forward, with the
    output assembled on every rank by the forward itself: q, k, v, g
    ([B, T, H_r, *]) and h0 ([B, H_r, K, V]) hold this rank's head range,
    and every chunk's O is TMA-stored from the kernel into block `rank` of
    every rank's `peers` buffer (PeerBuffers(world, width): block r = rank
    r's [B, T, H_r, V] output, width >= B*T*max(H_r)*V), over NVLink
    (gl_chunk_gla_fwd_scatter).  The same two stream-ordered all-reduces of
    one int as gmm_fp8_fwd_gathered order the stores after every rank's
    earlier work on its buffer and the readers after every rank's kernel.
    Returns `peers.local` ([world, width]): the shared buffer, valid until
    the next call.  Collective: every rank calls it, in the same order.
    Each head's computation is the single-GPU one, so the blocks equal a
    one-GPU forward of the same heads bit for bit."""
    import torch.distributed as dist
    from . import ops
    rank, world = dist.get_rank(), dist.get_world_size()
    B, T, Hr, V = v.shape
    if B * T * Hr * V > width or tuple(peers.local.shape) != (world, width):
        raise ValueError("peers must be PeerBuffers(world, width) with width >= B*T*H_r*V")
    if width % 8:  # every block must start 16-byte aligned
        raise ValueError("width must be a multiple of 8 elements")
    flag = torch.zeros(1, dtype=torch.int32, device=peers.local.device)
    dist.all_reduce(flag)
    outs = [p + rank * width * 2 for p in ring_order(peers.ptrs, rank)]
    ops.chunk_gla_fwd_scatter(q, k, v, None, scale, 64, outs=outs, g=g, h0=h0, ht=ht,
                              exact_intra=exact_intra)
    dist.all_reduce(flag)
    return peers.local
