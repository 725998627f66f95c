"""Sequence-sharded chunked decode over the GPUs of one node.

One process per GPU.  Rank ``r`` of ``N`` holds a contiguous range of the
context's chunks (its KV shard) and computes a partial ``(o, lse)`` over them
with the split-KV kernel.  The ``N`` partials (fp32, ``B*H*(D_v+1)`` values
per rank) are exchanged and folded on every rank: by default in one kernel
that stores each row into every peer's exchange buffer over NVLink (CUDA IPC
mappings, ``halo_sharded_decode``), or with an NCCL all-gather and the
LSE-merge kernel (``exchange="nccl"``).  The merge is associative and
commutative (the identity behind
``halo/kv_cache_chunked.py:194-239``; reference path relative to the
lzbaclz/HALO root), so the result equals single-GPU attention over the whole
context up to fp32 reduction order.  The reference runs on one GPU only; this
sharding is new.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from halo_b200 import ops


def shard_range(n_chunks: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous chunk range ``[lo, hi)`` owned by ``rank`` (balanced)."""
    base, extra = divmod(n_chunks, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_partials(o_local: torch.Tensor, lse_local: torch.Tensor, group=None,
                    buffers: Optional[tuple] = None):
    """All-gather every rank's partial ``(o (B, H, D_v), lse (B, H))``, fp32.

    One collective over a packed ``[o | lse]`` row per rank; returns
    ``(lse_parts (W, B, H), o_parts (W, B, H, D_v))`` in rank order -- views
    into the gathered buffer, laid out for ``ops.lse_merge(...,
    parts_major=True)``.  ``buffers = (local, gathered)`` reuses storage.
    Works with any ``torch.distributed`` backend (NCCL on GPUs, gloo in
    the CPU tests)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    B, H, D_v = o_local.shape
    R = B * H
    n = R * D_v + R
    if buffers is None:
        local = torch.empty(n, dtype=torch.float32, device=o_local.device)
        gathered = torch.empty(world * n, dtype=torch.float32, device=o_local.device)
    else:
        local, gathered = buffers
    if o_local.data_ptr() != local.data_ptr():
        local[:R * D_v].copy_(o_local.reshape(-1))
        local[R * D_v:].copy_(lse_local.reshape(-1))
    dist.all_gather_into_tensor(gathered, local, group=group)   # flat: gloo and NCCL
    rows = gathered.view(world, n)
    return rows[:, R * D_v:].view(world, B, H), rows[:, :R * D_v].view(world, B, H, D_v)


class P2PExchange:
    """Every rank's exchange buffer mapped in this process (CUDA IPC over
    NVLink), for ``halo_sharded_merge``.  Collective: every rank of `group`
    constructs it at the same point."""

    def __init__(self, rows: int, D_v: int, group=None):
        import torch.distributed as dist
        from halo_b200 import _lib as L
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        lib = L.lib()
        nbytes = lib.halo_exchange_bytes(self.world, rows, D_v)
        if nbytes < 0:
            L.check(int(nbytes), "halo_exchange_bytes")
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        L.check(lib.halo_ipc_alloc(nbytes, ctypes.byref(own), handle), "halo_ipc_alloc")
        self._own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs, self._opened = [], []
        for j, h in enumerate(handles):
            if j == self.rank:
                ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(h, 64)
            L.check(lib.halo_ipc_open(buf, ctypes.byref(p)), "halo_ipc_open")
            ptrs.append(p.value)
            self._opened.append(p.value)
        self.bufs = (ctypes.c_void_p * self.world)(*ptrs)
        torch.cuda.synchronize()
        dist.barrier(group)

    def close(self) -> None:
        from halo_b200 import _lib as L
        lib = L.lib()
        torch.cuda.synchronize()
        for p in self._opened:
            lib.halo_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        if self._own:
            lib.halo_ipc_free(ctypes.c_void_p(self._own))
            self._own = None


class ShardedDecoder:
    """Decode attention of a query over a sequence-sharded KV cache.

    ``k_shard`` / ``v_shard``: this rank's ``(B, H_kv, T_local, D)`` rows,
    whose first row sits at global position ``start``; they are attended in
    chunks of ``chunk_size`` (the chunk list is described once).  ``group`` is
    a ``torch.distributed`` process group (NCCL) or ``None`` for one GPU.
    ``exchange``: ``"p2p"`` merges across ranks with one fused kernel over
    NVLink peer memory (``halo_sharded_merge``), ``"nccl"`` with a local
    merge, an NCCL all-gather and a merge of the gathered parts.
    """

    def __init__(self, k_shard: torch.Tensor, v_shard: torch.Tensor, *, start: int = 0,
                 chunk_size: int = 4096, group=None, exchange: str = "p2p"):
        import torch.distributed as dist
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange must be 'p2p' or 'nccl', not {exchange!r}")
        self.k, self.v = k_shard, v_shard
        self.group = group
        self.exchange = exchange
        self._x = None
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
            gathered = torch.empty(self.world * (R * D_v + R), dtype=torch.float32, device=dev)
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
        if self.exchange == "p2p":
            return self._p2p_call(q3, scale, out, lse, events)
        R = B * H
        local, gathered = self._buffers(B, H, D_v, q3.device)
        o_loc, l_loc = local[:R * D_v].view(B, H, D_v), local[R * D_v:].view(B, H)
        ops.chunked_decode(q3, self.table, scale=scale, out=o_loc, lse=l_loc, events=events)
        m_parts, o_parts = gather_partials(o_loc, l_loc, self.group, buffers=(local, gathered))
        if out is None:
            out = torch.empty(B, H, D_v, dtype=q3.dtype, device=q3.device)
        return ops.lse_merge(m_parts, None, o_parts, out=out, lse=lse, parts_major=True)

    def _p2p_call(self, q3, scale, out, lse, events):
        B, H, D = q3.shape
        D_v = self.table.D_v
        if self._x is None or self._x_key != (B, H, D_v):
            if self._x is not None:
                self._x.close()
            self._x = P2PExchange(B * H, D_v, self.group)
            self._x_key = (B, H, D_v)
        if out is None:
            out = torch.empty(B, H, D_v, dtype=q3.dtype, device=q3.device)
        return ops.sharded_decode(q3, self.table, self._x, scale=scale, out=out, lse=lse,
                                  events=events)

    def capture(self, q: torch.Tensor, *, out: torch.Tensor, lse: Optional[torch.Tensor] = None,
                scale: Optional[float] = None) -> "torch.cuda.CUDAGraph":
        """Capture one call on the fixed buffers ``q``/``out``/``lse`` in a
        CUDA graph; ``graph.replay()`` reruns the decode on whatever ``q``
        holds, with no host work per step beyond the graph launch.  Makes
        one eager call first (plans, workspace, exchange buffers), so every
        rank must capture at the same point of its call sequence.  The
        cross-GPU exchange counts its epochs on the device, so replays stay
        in step across ranks.  ``exchange="nccl"`` is not captured (its
        collective runs through ``torch.distributed``).  The graph refers
        to this decoder's workspace and exchange buffers: release it before
        :meth:`close`."""
        if self.world > 1 and self.exchange != "p2p":
            raise ValueError("capture() needs exchange='p2p' when sharded")
        # the eager call runs on the capture stream so the stream's workspace
        # exists (zeroed) before capture
        side = torch.cuda.Stream(q.device)
        side.wait_stream(torch.cuda.current_stream(q.device))
        with torch.cuda.stream(side):
            self(q, out=out, lse=lse, scale=scale)
        torch.cuda.synchronize(q.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            self(q, out=out, lse=lse, scale=scale)
        return graph

    def close(self) -> None:
        """Release the peer mappings (collective-free; call on every rank)."""
        if self._x is not None:
            self._x.close()
            self._x = None

    @property
    def launches_per_call(self) -> int:
        """Kernels of this library per call, as counted by
        ``halo_launch_count``: split-KV + merge on one GPU, split-KV +
        exchange merge (p2p) or split-KV + local merge + merge of the
        gathered parts (nccl) when sharded."""
        if self.world == 1:
            return 2
        return 2 if self.exchange == "p2p" else 3


class ShardedKiviDecoder:
    """KIVI decode over a sequence-sharded quantised cache (the packed
    2/4/8-bit format of ``baselines.kivi_cache``; the reference's KIVI cache,
    ``baselines/kivi_cache.py:121-195``, is single-GPU).

    Rank ``r`` quantises and holds its contiguous rows ``k_shard`` /
    ``v_shard`` ``(B, H_kv, T_local, D)`` (``T_local`` a multiple of
    ``group_size``; quantisation is per row, so the codes equal those a
    single cache would hold for the same rows); the rank holding the end of
    the context may also pass the most recent rows in 16 bits
    (``recent_k`` / ``recent_v``).  A call attends this rank's rows with the
    fused packed kernel (and the recent rows with the split-KV kernel, folded
    in by LSE), then merges every rank's normalised fp32 ``(o, lse)``:
    ``exchange="p2p"`` in one kernel over NVLink peer memory
    (``halo_sharded_merge`` with one normalised part per rank), ``"nccl"``
    with an all-gather and the merge kernel, as :class:`ShardedDecoder`.
    The keys are not causal-masked against each other: every cached row
    precedes the decode query.
    """

    def __init__(self, k_shard: torch.Tensor, v_shard: torch.Tensor, *, bits: int = 2,
                 group_size: int = 32, recent_k: Optional[torch.Tensor] = None,
                 recent_v: Optional[torch.Tensor] = None, group=None,
                 exchange: str = "p2p"):
        import torch.distributed as dist
        from halo_b200.baselines.kivi_cache import _Packed
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange must be 'p2p' or 'nccl', not {exchange!r}")
        self.exchange = exchange
        self._x = None
        if k_shard.shape[-2] % group_size:
            raise ValueError("rows per shard must be a multiple of group_size")
        self.group = group
        self.world = dist.get_world_size(group) if (group is not None or (
            dist.is_available() and dist.is_initialized())) else 1
        self.bits = bits
        B, H_kv, T, D = k_shard.shape
        self.kq = _Packed(B, H_kv, D, k_shard.dtype, k_shard.device, bits, group_size)
        self.vq = _Packed(B, H_kv, v_shard.shape[-1], v_shard.dtype, v_shard.device, bits,
                          group_size)
        if T:
            self.kq.append(k_shard)
            self.vq.append(v_shard)
        self.recent = []
        if recent_k is not None and recent_k.shape[-2]:
            self.recent = [(recent_k, recent_v, 0, False)]
        self._bufs: dict = {}

    def _buffers(self, B: int, H: int, D_v: int, dev: torch.device):
        key = (B, H, D_v)
        if key not in self._bufs:
            R = B * H
            local = torch.empty(R * D_v + R, dtype=torch.float32, device=dev)
            gathered = torch.empty(self.world * (R * D_v + R), dtype=torch.float32, device=dev)
            ones = torch.ones(B, H, dtype=torch.float32, device=dev)
            self._bufs[key] = (local, gathered, ones)
        return self._bufs[key]

    def __call__(self, q: torch.Tensor, *, scale: Optional[float] = None,
                 out: Optional[torch.Tensor] = None):
        """``q (B, H, D)`` or ``(B, H, 1, D)``; returns ``(out (B, H, D_v) in
        q.dtype, lse (B, H) fp32)`` over the rows of every rank."""
        from halo_b200.baselines.kivi_cache import kivi_decode
        q3 = q.squeeze(2) if q.dim() == 4 else q
        q3 = q3 if q3.is_contiguous() else q3.contiguous()
        B, H, D = q3.shape
        D_v = self.vq.D
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        R = B * H
        local, gathered, ones = self._buffers(B, H, D_v, q3.device)
        o_loc, l_loc = local[:R * D_v].view(B, H, D_v), local[R * D_v:].view(B, H)
        if self.kq.T:
            if self.recent:
                o_p = torch.empty(B, H, D_v, dtype=torch.float32, device=q3.device)
                l_p = torch.empty(B, H, dtype=torch.float32, device=q3.device)
                kivi_decode(q3, self.kq, self.vq, self.kq.T, self.bits, scale=scale, out=o_p,
                            lse=l_p)
                ops.chunked_decode(q3, self.recent, scale=scale, out=o_loc, lse=l_loc,
                                   prior=(l_p, ones, o_p))
            else:
                kivi_decode(q3, self.kq, self.vq, self.kq.T, self.bits, scale=scale, out=o_loc,
                            lse=l_loc)
        elif self.recent:
            ops.chunked_decode(q3, self.recent, scale=scale, out=o_loc, lse=l_loc)
        else:
            # no rows on this rank: a part that the merge gives zero weight
            o_loc.zero_()
            l_loc.fill_(float("-inf"))
        if out is None:
            out = torch.empty(B, H, D_v, dtype=q3.dtype, device=q3.device)
        if self.world == 1:
            out.copy_(o_loc)
            return out, l_loc.clone()
        if self.exchange == "p2p":
            return self._p2p_merge(o_loc, l_loc, out)
        m_parts, o_parts = gather_partials(o_loc, l_loc, self.group, buffers=(local, gathered))
        return ops.lse_merge(m_parts, None, o_parts, out=out, parts_major=True)

    def _p2p_merge(self, o_loc: torch.Tensor, l_loc: torch.Tensor, out: torch.Tensor):
        from halo_b200 import _lib as L
        B, H, D_v = o_loc.shape
        if self._x is None or self._x_key != (B, H, D_v):
            if self._x is not None:
                self._x.close()
            self._x = P2PExchange(B * H, D_v, self.group)
            self._x_key = (B, H, D_v)
        lse = torch.empty(B, H, dtype=torch.float32, device=o_loc.device)
        # one normalised part per rank: m = its lse, l = 1 (NULL), o = its out
        with torch.cuda.device(o_loc.device):
            rc = L.lib().halo_sharded_merge(
                B, H, D_v, 1, l_loc.data_ptr(), None, o_loc.data_ptr(), 1, 1, D_v, D_v,
                self._x.world, self._x.rank, self._x.bufs, L.halo_dtype(out.dtype),
                out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
                L.stream_handle(o_loc.device))
        L.check(rc, "halo_sharded_merge")
        return out, lse

    def close(self) -> None:
        """Release the peer mappings (call on every rank)."""
        if self._x is not None:
            self._x.close()
            self._x = None
