"""Multi-GPU partitioning of the op set (one process per GPU, torch.distributed).

Every op shards without communication on its data path:
  * attention over batch x heads, quantisation over rows, the GEMMs over tokens (rows of A /
    x) with replicated weights -> ``shard_range`` / ``shard_rows``;
  * optionally a weight is split by output columns (N / g per rank) and the ``[M, N/g]``
    partial outputs are gathered into a replicated ``[M, N]`` with one
    ``all_gather_into_tensor`` -> ``shard_columns`` / ``gather_columns`` /
    ``column_sharded_int8_linear``.
The gather is the only collective; it runs over NCCL on GPUs and over gloo in the CPU tests.

``column_sharded_int8_linear_fused`` does the same layer with the gather inside the GEMM: each
rank's epilogue stores its ``[M, N/g]`` tiles straight into every rank's replicated output
(``PeerBuffers``: the peers' buffers mapped into this process with CUDA IPC, written over
NVLink), so the transfer overlaps the GEMM tile by tile; two one-element NCCL all-reduces
order the launch against the buffers' other users.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = [
    "shard_range",
    "shard_rows",
    "gather_rows",
    "shard_columns",
    "gather_columns",
    "column_sharded_int8_linear",
    "PeerBuffers",
    "column_sharded_int8_linear_fused",
    "MulticastBuffers",
    "column_sharded_int8_linear_multicast",
]


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, stop) of ``n`` items for ``rank`` of ``world``; sizes differ by <= 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n < 0:
        raise ValueError("n must be >= 0")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_rows(t: torch.Tensor, rank: int, world: int, dim: int = 0) -> torch.Tensor:
    """This rank's slice of ``t`` along ``dim`` (a view, no copy)."""
    s, e = shard_range(t.shape[dim], rank, world)
    return t.narrow(dim, s, e - s)


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def gather_rows(local: torch.Tensor, total_rows: int, group=None) -> torch.Tensor:
    """Inverse of ``shard_rows`` along dim 0: every rank receives the full tensor.  Uneven
    shards are padded to the largest shard for the collective and trimmed afterwards."""
    world, _ = _world(group)
    cap = -(-total_rows // world)
    pad = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]].copy_(local)
    out = torch.empty((world * cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, pad, group=group)
    pieces = []
    for r in range(world):
        s, e = shard_range(total_rows, r, world)
        pieces.append(out[r * cap: r * cap + (e - s)])
    return torch.cat(pieces, 0)


def shard_columns(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Output-column shard of a weight stored ``[N, K]`` (its rows), contiguous."""
    return shard_rows(w, rank, world, 0).contiguous()


def gather_columns(local: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """``[M, N_r]`` per rank -> replicated ``[M, n_total]`` with rank r's columns at its
    ``shard_range``.  One ``all_gather_into_tensor`` of equal-sized (padded) blocks."""
    world, _ = _world(group)
    M = local.shape[0]
    cap = -(-n_total // world)
    blk = torch.zeros((M, cap), dtype=local.dtype, device=local.device)
    blk[:, : local.shape[1]].copy_(local)
    out = torch.empty((world, M, cap), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out.view(world * M, cap), blk, group=group)
    cols = []
    for r in range(world):
        s, e = shard_range(n_total, r, world)
        cols.append(out[r, :, : e - s])
    return torch.cat(cols, 1)


def column_sharded_int8_linear(x: torch.Tensor, w_q_shard: torch.Tensor, scale_w_shard: torch.Tensor,
                               n_total: int, group=None, replicate: bool = True) -> torch.Tensor:
    """Tensor-parallel ``Int8Linear`` forward: quantise ``x`` (replicated), multiply by this
    rank's ``[N/g, K]`` weight shard with the sm_100a int8 GEMM, then (``replicate=True``)
    gather the ``[M, N/g]`` fp16 blocks into ``[M, N]`` on every rank."""
    from .int8_gemm import int8_gemm_dequant_nk, quantize_symmetric

    xq, sx = quantize_symmetric(x)
    y = int8_gemm_dequant_nk(xq, w_q_shard, sx, scale_w_shard)
    return gather_columns(y, n_total, group) if replicate else y


class PeerBuffers:
    """One ``shape`` fp16 buffer per rank of ``group`` (one process per GPU), with every
    peer's buffer mapped into this process: ``ptrs[r]`` is the device address of rank r's
    buffer as seen from this rank's GPU (``ptrs[rank]`` is ``local``'s own address).  Kernels
    on this GPU may store into all of them; NVLink carries the stores to the peers.

    Collective: every rank constructs it with the same shape, in the same order.  Call
    ``close()`` (also collective) before the process group is destroyed."""

    def __init__(self, shape, group=None, dtype=torch.float16):
        import ctypes

        from . import _lib

        world, rank = _world(group)
        self.group, self.rank, self.world = group, rank, world
        self.device = torch.cuda.current_device()
        self.local = torch.empty(shape, dtype=dtype, device=f"cuda:{self.device}")
        handle = (ctypes.c_char * _lib.LK_PEER_HANDLE_BYTES)()
        off = ctypes.c_int64()
        _lib.call("lk_peer_export", self.device, ctypes.c_void_p(self.local.data_ptr()), handle, ctypes.byref(off))
        infos = [None] * world
        dist.all_gather_object(infos, (bytes(handle), off.value), group=group)
        self._opened = []
        self.ptrs = []
        for r in range(world):
            if r == rank:
                self.ptrs.append(self.local.data_ptr())
                continue
            h, o = infos[r]
            p = ctypes.c_void_p()
            _lib.call("lk_peer_open", self.device, ctypes.create_string_buffer(h, len(h)), o, ctypes.byref(p))
            self.ptrs.append(p.value)
            self._opened.append((p.value, o))

    def close(self):
        """Unmaps the peers' buffers once every rank is done with them (collective)."""
        from . import _lib

        if self._opened is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p, o in self._opened:
            _lib.call("lk_peer_close", self.device, p, o)
        self._opened = None


def column_sharded_int8_linear_fused(x: torch.Tensor, w_q_shard: torch.Tensor, scale_w_shard: torch.Tensor,
                                     out: PeerBuffers, group=None) -> torch.Tensor:
    """``column_sharded_int8_linear`` with the gather fused into the GEMM epilogue.

    ``out`` is a ``PeerBuffers`` of shape ``[M, N_total]``; rank r's columns are its
    ``shard_range(N_total, r, g)`` and must start at a multiple of 8 (N_total a multiple of
    8 * g does it).  Returns ``out.local``, the replicated ``[M, N_total]`` fp16 result, valid
    on the current stream.  The all-reduce before the launch is ordered after the work already
    queued on each rank's CURRENT stream, so it keeps a rank from overwriting a peer's buffer
    while the peer's current stream still reads it; the one after it completes only when every
    rank's stores have landed.  Every reader of ``out.local`` (and of an earlier result held in
    it) must therefore run on the calling stream, or be ordered before this call on it (e.g. by
    an event the caller records on its side stream and makes the current stream wait for):
    peers' stores are not ordered against work on other streams."""
    from .int8_gemm import int8_gemm_dequant_scatter, quantize_symmetric

    world, rank = _world(group)
    M, n_total = out.local.shape
    s, e = shard_range(n_total, rank, world)
    if w_q_shard.shape[0] != e - s:
        raise ValueError(f"rank {rank}: weight shard has {w_q_shard.shape[0]} rows, expected {e - s}")
    if s % 8:
        raise ValueError("column blocks must start at multiples of 8 (N_total a multiple of 8 * world)")
    xq, sx = quantize_symmetric(x)
    flag = torch.zeros(1, device=x.device)
    dist.all_reduce(flag, group=group)
    int8_gemm_dequant_scatter(xq, w_q_shard, sx, scale_w_shard, out.ptrs, n_total, s)
    dist.all_reduce(flag, group=group)
    return out.local


class MulticastBuffers:
    """One ``shape`` fp16 buffer per rank of ``group`` in torch symmetric memory, bound to an
    NVLink multicast object: a store to ``multicast_ptr`` (a multimem store, issued once by one
    GPU) is written by the NVSwitch into every rank's buffer.  ``local`` is this rank's buffer.

    Collective: every rank constructs it with the same shape, in the same order.  Raises
    ``RuntimeError`` where the GPUs have no multicast support (no NVSwitch / NVLS).  ``close()``
    (collective) before the process group is destroyed."""

    def __init__(self, shape, group=None, dtype=torch.float16):
        import torch.distributed._symmetric_memory as symm_mem

        group = group if group is not None else dist.group.WORLD
        self.group = group
        self.world, self.rank = _world(group)
        self.device = torch.cuda.current_device()
        self.local = symm_mem.empty(*shape, dtype=dtype, device=f"cuda:{self.device}")
        self.handle = symm_mem.rendezvous(self.local, group)
        if not self.handle.multicast_ptr:
            raise RuntimeError("NVLink multicast is not available on these GPUs")
        # The tensor's place inside its symmetric allocation, applied to the multicast base.
        offset = self.local.data_ptr() - self.handle.buffer_ptrs[self.rank]
        self.multicast_ptr = self.handle.multicast_ptr + offset

    def barrier(self):
        """Device-side barrier of all ranks on the current stream (symmetric-memory signals)."""
        self.handle.barrier()

    def close(self):
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.handle = None
        self.local = None


def column_sharded_int8_linear_multicast(x: torch.Tensor, w_q_shard: torch.Tensor, scale_w_shard: torch.Tensor,
                                         out: "MulticastBuffers", group=None) -> torch.Tensor:
    """``column_sharded_int8_linear`` with the gather done by the NVSwitch: the GEMM epilogue
    stores each tile of this rank's ``[M, N/g]`` block once to ``out.multicast_ptr`` and the
    switch replicates it into every rank's ``[M, N_total]`` output, so each rank's block crosses
    NVLink once (the peer-store path sends it once per peer).  Per-rank column blocks must be
    multiples of 32 wide and start at multiples of 8.  Returns ``out.local``; a device barrier
    before the launch keeps a rank from overwriting outputs its peers still read on their
    current streams, one after it completes once every rank's stores have landed (the same
    ordering contract as ``column_sharded_int8_linear_fused``)."""
    from .int8_gemm import int8_gemm_dequant_multicast, quantize_symmetric

    world, rank = _world(group)
    M, n_total = out.local.shape
    s, e = shard_range(n_total, rank, world)
    if w_q_shard.shape[0] != e - s:
        raise ValueError(f"rank {rank}: weight shard has {w_q_shard.shape[0]} rows, expected {e - s}")
    if s % 8 or (e - s) % 32:
        raise ValueError("column blocks must start at multiples of 8 and be multiples of 32 wide")
    xq, sx = quantize_symmetric(x)
    out.barrier()
    int8_gemm_dequant_multicast(xq, w_q_shard, sx, scale_w_shard, out.multicast_ptr, n_total, s)
    out.barrier()
    return out.local
