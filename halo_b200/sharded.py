"""Sequence-sharded chunked decode over the GPUs of one node.

One process per GPU.  Rank ``r`` of ``N`` holds a contiguous range of the
context's chunks (its KV shard) and computes a partial ``(o, lse)`` over them
with the split-KV kernel; the ``N`` partials (fp32, ``B*H*(D_v+1)`` floats per
rank) are all-gathered over NCCL and folded by the LSE-merge kernel on every
rank.  The merge is associative and commutative (the identity behind
``halo/kv_cache_chunked.py:194-239``; reference path relative to the
lzbaclz/HALO root), so the result equals single-GPU attention over the whole
context up to fp32 reduction order.  The reference runs on one GPU only; this
sharding is new.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from halo_b200 import ops


def shard_range(n_chunks: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous chunk range ``[lo, hi)`` owned by ``rank`` (balanced)."""
    base, extra = divmod(n_chunks, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


class ShardedDecoder:
    """Decode attention of a query over a sequence-sharded KV cache.

    ``k_shard`` / ``v_shard``: this rank's ``(B, H_kv, T_local, D)`` rows,
    whose first row sits at global position ``start``; they are attended in
    chunks of ``chunk_size`` (the chunk list is described once).  ``group`` is
    a ``torch.distributed`` process group (NCCL) or ``None`` for one GPU.
    """

    def __init__(self, k_shard: torch.Tensor, v_shard: torch.Tensor, *, start: int = 0,
                 chunk_size: int = 4096, group=None):
        import torch.distributed as dist
        self.k, self.v = k_shard, v_shard
        self.group = group
        self.world = dist.get_world_size(group) if (group is not None or (
            dist.is_available() and dist.is_initialized())) else 1
        T = k_shard.shape[-2]
        self.chunks = [(k_shard[..., a:min(a + chunk_size, T), :],
                        v_shard[..., a:min(a + chunk_size, T), :], start + a, False)
                       for a in range(0, T, chunk_size)]
        self.table = ops.ChunkTable(self.chunks)
        self._bufs: dict = {}

    def _buffers(self, B: int, H: int, D_v: int, dev: torch.device):
        key = (B, H, D_v)
        if key not in self._bufs:
            R = B * H
            local = torch.empty(R * D_v + R, dtype=torch.float32, device=dev)
            gathered = torch.empty(self.world, R * D_v + R, dtype=torch.float32, device=dev)
            self._bufs[key] = (local, gathered)
        return self._bufs[key]

    def __call__(self, q: torch.Tensor, *, scale: Optional[float] = None,
                 out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
                 events: Optional[tuple] = None):
        """Returns ``(out (B, H, D_v) in q.dtype, lse (B, H) fp32)``."""
        q3 = q.squeeze(2) if q.dim() == 4 else q
        B, H, D = q3.shape
        D_v = self.table.D_v
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        if self.world == 1:
            return ops.chunked_decode(q3, self.table, scale=scale, out=out, lse=lse,
                                      events=events)
        import torch.distributed as dist
        R = B * H
        local, gathered = self._buffers(B, H, D_v, q3.device)
        ops.chunked_decode(q3, self.table, scale=scale,
                           out=local[:R * D_v].view(B, H, D_v), lse=local[R * D_v:].view(B, H),
                           events=events)
        dist.all_gather_into_tensor(gathered, local, group=self.group)
        m_parts = gathered[:, R * D_v:].view(self.world, B, H)
        o_parts = gathered[:, :R * D_v].view(self.world, B, H, D_v)
        if out is None:
            out = torch.empty(B, H, D_v, dtype=q3.dtype, device=q3.device)
        return ops.lse_merge(m_parts, None, o_parts, out=out, lse=lse, parts_major=True)

    @property
    def launches_per_call(self) -> int:
        """Kernels of this library per call (split-KV, local merge, and the
        cross-rank merge when sharded)."""
        return 2 + (1 if self.world > 1 else 0)
