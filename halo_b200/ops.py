"""Tensor-level entry points over the C-ABI (``include/halo_b200.h``).

Every function here launches sm_100a kernels from ``libhalo_sm100.so`` on the
current CUDA stream; there is no CPU path.  Tensors follow the reference's
layouts: queries ``(B, H, D)`` / ``(B, H, T_q, D)`` and K/V chunks
``(B, H_kv, T_c, D)`` with a contiguous last dimension.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence

import torch

from halo_b200 import _lib as L


class _Workspaces:
    """Grow-only device scratch per (device, stream); stream-ordered reuse.
    Allocated zeroed: the decode workspaces start with a control block that
    must be zero before first use (the kernels leave it zero)."""

    def __init__(self):
        self._bufs: dict = {}

    def get(self, device: torch.device, nbytes: int, stream: Optional[int] = None) -> torch.Tensor:
        """``stream``: the raw handle of the stream the buffer is used on
        (default: ``device``'s current stream)."""
        if stream is None:
            stream = L.stream_handle(device)
        key = (device.index, stream)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf


WORKSPACES = _Workspaces()
# prefill's staging workspace (fp16 copies of V): kept apart from the decode
# workspaces, whose leading control block must stay zero between calls
PREFILL_WORKSPACES = _Workspaces()


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise L.HaloError(f"{name} must be a CUDA tensor (no CPU path)", L.HALO_ERR_INVALID_ARG)


def _last_contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def make_chunk(k: torch.Tensor, v: torch.Tensor, start: int, causal: bool,
               *, batch_stride_zero: bool = False) -> tuple:
    """Describe one ``(B, H_kv, T_c, D)`` chunk for the C-ABI; returns the
    struct plus the tensors it points into (keep them alive)."""
    k = _last_contig(k)
    v = _last_contig(v)
    c = L.KVChunk()
    c.k = k.data_ptr() if k.numel() else None
    c.v = v.data_ptr() if v.numel() else None
    c.k_stride_b = 0 if batch_stride_zero else k.stride(0)
    c.k_stride_h, c.k_stride_t = k.stride(1), k.stride(2)
    c.v_stride_b = 0 if batch_stride_zero else v.stride(0)
    c.v_stride_h, c.v_stride_t = v.stride(1), v.stride(2)
    c.start = int(start)
    c.len = int(k.shape[2]) if k.numel() else 0
    c.causal = int(bool(causal))
    return c, (k, v)


def _problem(q3: torch.Tensor, H_kv: int, D_v: int, q_pos: Optional[torch.Tensor], scale: float,
             max_split_rows: int = 0) -> L.DecodeProblem:
    p = L.DecodeProblem()
    p.B, p.H, p.D = q3.shape
    p.H_kv = H_kv
    p.Dv = D_v
    p.dtype = L.halo_dtype(q3.dtype)
    p.q = q3.data_ptr()
    p.q_stride_b, p.q_stride_h = q3.stride(0), q3.stride(1)
    p.q_pos = q_pos.data_ptr() if q_pos is not None else None
    p.scale = float(scale)
    p.max_split_rows = int(max_split_rows)
    return p


def decode_raw(q3: torch.Tensor, chunk_structs: Sequence[L.KVChunk], H_kv: int, D_v: int, *,
               scale: float, q_pos: Optional[torch.Tensor], merge: L.MergeArgs,
               max_split_rows: int = 0) -> None:
    """Launch split-KV decode + merge for prepared chunk structs."""
    dev = q3.device
    prob = _problem(q3, H_kv, D_v, q_pos, scale, max_split_rows)
    n = len(chunk_structs)
    arr = (L.KVChunk * max(n, 1))(*chunk_structs)
    lib = L.lib()
    need = lib.halo_decode_workspace_bytes(ctypes.byref(prob), arr, n)
    if need < 0:
        L.check(int(need), "halo_decode_workspace_bytes")
    sh = L.stream_handle(dev)
    ws = WORKSPACES.get(dev, int(need), sh)
    with L.on_device(dev):
        rc = lib.halo_chunked_decode(ctypes.byref(prob), arr, n, ws.data_ptr(), ws.numel(),
                                     ctypes.byref(merge), sh)
    L.check(rc, "halo_chunked_decode")


class ChunkTable:
    """A chunk list described once for repeated decode calls.

    Holds the C-ABI chunk array and references to the tensors it points
    into.  Reuse it while the chunks' storage and layout stay unchanged (the
    steady state of a decode loop); the library additionally memoises the
    tensor maps and the split plan for a layout it has seen.
    """

    def __init__(self, chunks: Sequence[tuple], *, batch_stride_zero: bool = False,
                 batch: Optional[slice] = None):
        structs, keep = [], []
        self.H_kv = self.D_v = None
        self.total_rows = 0
        self.any_causal = False
        for (k, v, start, causal) in chunks:
            _require_cuda(k, "k")
            _require_cuda(v, "v")
            if batch is not None:
                k, v = k[batch], v[batch]
            if self.H_kv is None:
                self.H_kv, self.D_v = int(k.shape[1]), int(v.shape[-1])
            st, t = make_chunk(k, v, start, causal, batch_stride_zero=batch_stride_zero)
            structs.append(st)
            keep.append(t)
            self.total_rows += int(k.shape[-2])
            self.any_causal |= bool(causal)
        self.n = len(structs)
        self.arr = (L.KVChunk * max(self.n, 1))(*structs)
        self._keep = keep


def _decode_table(q3: torch.Tensor, table: ChunkTable, *, scale: float,
                  q_pos: Optional[torch.Tensor], merge: L.MergeArgs, max_split_rows: int = 0,
                  events: Optional[tuple] = None):
    dev = q3.device
    H_kv = table.H_kv if table.H_kv is not None else q3.shape[1]
    D_v = table.D_v if table.D_v is not None else q3.shape[2]
    prob = _problem(q3, H_kv, D_v, q_pos, scale, max_split_rows)
    if events is not None:
        prob.event_begin, prob.event_end = events
    lib = L.lib()
    need = lib.halo_decode_workspace_bytes(ctypes.byref(prob), table.arr, table.n)
    if need < 0:
        L.check(int(need), "halo_decode_workspace_bytes")
    sh = L.stream_handle(dev)
    ws = WORKSPACES.get(dev, int(need), sh)
    with L.on_device(dev):
        rc = lib.halo_chunked_decode(ctypes.byref(prob), table.arr, table.n, ws.data_ptr(),
                                     ws.numel(), ctypes.byref(merge), sh)
    L.check(rc, "halo_chunked_decode")


def decode_partials(q3: torch.Tensor, table: ChunkTable, *, scale: float,
                    q_pos: Optional[torch.Tensor] = None, events: Optional[tuple] = None):
    """Split-KV launches only (``halo_chunked_decode_partials``): returns
    ``(workspace, S, (m_off, l_off, o_off))`` -- the per-split fp32 partial
    state left in the workspace, ``m``/``l`` ``[B*H][S]``, ``o``
    ``[B*H][S][D_v]`` at those byte offsets -- for a caller-side merge."""
    dev = q3.device
    H_kv = table.H_kv if table.H_kv is not None else q3.shape[1]
    D_v = table.D_v if table.D_v is not None else q3.shape[2]
    prob = _problem(q3, H_kv, D_v, q_pos, scale)
    if events is not None:
        prob.event_begin, prob.event_end = events
    lib = L.lib()
    need = lib.halo_decode_workspace_bytes(ctypes.byref(prob), table.arr, table.n)
    if need < 0:
        L.check(int(need), "halo_decode_workspace_bytes")
    sh = L.stream_handle(dev)
    ws = WORKSPACES.get(dev, int(need), sh)
    n_parts = ctypes.c_int32(0)
    offs = (ctypes.c_int64 * 3)()
    with L.on_device(dev):
        rc = lib.halo_chunked_decode_partials(ctypes.byref(prob), table.arr, table.n,
                                              ws.data_ptr(), ws.numel(), ctypes.byref(n_parts),
                                              offs, sh)
    L.check(rc, "halo_chunked_decode_partials")
    return ws, int(n_parts.value), (int(offs[0]), int(offs[1]), int(offs[2]))


def sharded_decode(q3: torch.Tensor, table: ChunkTable, exchange, *, scale: float,
                   out: torch.Tensor, lse: Optional[torch.Tensor] = None,
                   q_pos: Optional[torch.Tensor] = None, events: Optional[tuple] = None):
    """One sequence-sharded decode step on this rank (``halo_sharded_decode``):
    attention over this rank's chunks merged with every rank's through the
    NVLink exchange buffers of ``exchange`` (a :class:`halo_b200.sharded.
    P2PExchange`).  Writes ``out (B, H, D_v)`` and ``lse (B, H)``."""
    dev = q3.device
    H_kv = table.H_kv if table.H_kv is not None else q3.shape[1]
    D_v = table.D_v if table.D_v is not None else q3.shape[2]
    prob = _problem(q3, H_kv, D_v, q_pos, scale)
    if events is not None:
        prob.event_begin, prob.event_end = events
    lib = L.lib()
    need = lib.halo_decode_workspace_bytes(ctypes.byref(prob), table.arr, table.n)
    if need < 0:
        L.check(int(need), "halo_decode_workspace_bytes")
    sh = L.stream_handle(dev)
    ws = WORKSPACES.get(dev, int(need), sh)
    with L.on_device(dev):
        rc = lib.halo_sharded_decode(ctypes.byref(prob), table.arr, table.n, ws.data_ptr(),
                                     ws.numel(), exchange.world, exchange.rank, exchange.bufs,
                                     L.halo_dtype(out.dtype), out.data_ptr(), out.stride(0),
                                     out.stride(1), lse.data_ptr() if lse is not None else None,
                                     sh)
    L.check(rc, "halo_sharded_decode")
    return out, lse


def chunked_decode(q: torch.Tensor, chunks, *, scale: Optional[float] = None,
                   q_pos: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                   out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
                   prior: Optional[tuple] = None, max_split_rows: int = 0,
                   events: Optional[tuple] = None, want_lse: bool = True):
    """Attention of one decode query over ``chunks`` -- a list of
    ``(k, v, start, causal)`` tuples or a prepared :class:`ChunkTable` --
    merged with log-sum-exp.  Returns ``(out (B, H, D_v), lse (B, H))``;
    with ``want_lse=False`` and no ``lse`` given, the log-sum-exp is not
    written and ``None`` is returned in its place.

    ``prior = (m, l, o)`` folds a running fp32 state in first.  ``q_pos``
    (device int64 ``(B,)``) defaults to ``total_T - 1`` as in
    ``halo/triton_chunked.py:250-253`` (reference path relative to the
    lzbaclz/HALO root).  ``events = (begin, end)`` are raw ``cudaEvent_t``
    handles recorded around the split-KV kernel launches (profiling).
    """
    q3 = q.squeeze(2) if q.dim() == 4 else q
    _require_cuda(q3, "q")
    q3 = q3 if q3.is_contiguous() else q3.contiguous()
    B, H, D = q3.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    table = chunks if isinstance(chunks, ChunkTable) else ChunkTable(chunks)
    D_v = table.D_v if table.D_v is not None else D
    if q_pos is None and table.any_causal:
        q_pos = torch.full((B,), table.total_rows - 1, dtype=torch.int64, device=q3.device)
    elif q_pos is not None and (q_pos.dtype != torch.int64 or q_pos.device != q3.device):
        q_pos = q_pos.to(device=q3.device, dtype=torch.int64).contiguous()
    if out is None:
        out = torch.empty(B, H, D_v, dtype=out_dtype or q3.dtype, device=q3.device)
    if lse is None and want_lse:
        lse = torch.empty(B, H, dtype=torch.float32, device=q3.device)
    mg = L.MergeArgs()
    mg.mode = L.MERGE_FINALIZE
    mg.out_dtype = L.halo_dtype(out.dtype)
    mg.out = out.data_ptr()
    mg.out_stride_b, mg.out_stride_h = out.stride(0), out.stride(1)
    mg.lse = lse.data_ptr() if lse is not None else None
    if prior is not None:
        m, l, o = prior
        mg.m, mg.l, mg.o = m.data_ptr(), l.data_ptr(), o.data_ptr()
    _decode_table(q3, table, scale=scale, q_pos=q_pos, merge=mg, max_split_rows=max_split_rows,
                  events=events)
    return out, lse


def accumulate_decode(q: torch.Tensor, chunks: Sequence[tuple], m: torch.Tensor, l: torch.Tensor,
                      o: torch.Tensor, *, scale: float, q_pos: Optional[torch.Tensor]) -> None:
    """Fold ``chunks`` into running fp32 accumulators ``(m, l, o)`` in place
    (the state ``update_chunk`` of ``halo/triton_chunked.py:151-192`` keeps)."""
    q3 = _last_contig(q.squeeze(2) if q.dim() == 4 else q)
    _require_cuda(q3, "q")
    for t, name in ((m, "m"), (l, "l"), (o, "o")):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise L.HaloError(f"accumulator {name} must be contiguous fp32", L.HALO_ERR_INVALID_ARG)
    structs, keep = [], []
    H_kv, D_v = q3.shape[1], o.shape[-1]
    for (k, v, start, causal) in chunks:
        H_kv, D_v = int(k.shape[1]), int(v.shape[-1])
        s, t = make_chunk(k, v, start, causal)
        structs.append(s)
        keep.append(t)
    if q_pos is not None:
        q_pos = q_pos.to(device=q3.device, dtype=torch.int64).contiguous()
    mg = L.MergeArgs()
    mg.mode = L.MERGE_ACCUMULATE
    mg.m, mg.l, mg.o = m.data_ptr(), l.data_ptr(), o.data_ptr()
    decode_raw(q3, structs, H_kv, D_v, scale=scale, q_pos=q_pos, merge=mg)


PREFILL_MAX_CHUNKS = 48   # chunk descriptors per halo_prefill_attention call


def prefill_supported(q: torch.Tensor, chunks: Sequence[tuple], scale: Optional[float] = None) -> bool:
    """Whether the tensor-core prefill kernel covers this problem: bf16 or
    fp16, head dim 64 or 128, value head dim equal to it, positive scale."""
    D = q.shape[-1]
    if q.dtype not in (torch.bfloat16, torch.float16) or D not in (64, 128):
        return False
    if scale is not None and not (math.isfinite(scale) and scale > 0):
        return False
    return all(k.dtype == q.dtype and v.dtype == q.dtype and k.shape[-1] == D and
               v.shape[-1] == D for (k, v, _s, _c) in chunks)


def prefill_attention(q: torch.Tensor, chunks: Sequence[tuple], *, query_pos_offset: int,
                      scale: Optional[float] = None, out_dtype: Optional[torch.dtype] = None,
                      out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
                      state: Optional[tuple] = None, accumulate: bool = False,
                      events: Optional[tuple] = None):
    """Chunked-prefill attention on the tcgen05 kernel
    (``halo_prefill_attention_ws``): ``q (B, H, T_q, D)`` with query row ``i``
    at global position ``query_pos_offset + i`` over ``(k, v, start, causal)``
    chunks (``halo/kv_cache_chunked.py:873-942``).

    ``state = (m, l, o)``: fp32 running state, ``m, l (B, H, T_q)`` and
    ``o (B, H, T_q, D)`` contiguous.  ``accumulate=True`` folds the chunks
    into it in place and returns ``None``; otherwise the state (if given) is
    folded in and ``(out (B, H, T_q, D), lse (B, H, T_q))`` is returned, and
    the caller's state is left as it was.  Lists longer than one call takes
    (more than ``PREFILL_MAX_CHUNKS`` non-contiguous chunks) run as several
    calls through a running state of their own."""
    _require_cuda(q, "q")
    B, H, T_q, D = q.shape
    if q.stride(-1) != 1:
        q = q.contiguous()
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    H_kv = int(chunks[0][0].shape[1]) if chunks else H
    groups = [chunks[i:i + PREFILL_MAX_CHUNKS] for i in range(0, len(chunks), PREFILL_MAX_CHUNKS)]
    if not groups:
        groups = [[]]
    if accumulate and state is None:
        raise L.HaloError("accumulate needs state=(m, l, o)", L.HALO_ERR_INVALID_ARG)
    if len(groups) > 1 and not accumulate:
        # the groups fold into a state of this call's own (a copy of the
        # caller's, if given): the caller's tensors are only read
        if state is None:
            state = (torch.full((B, H, T_q), float("-inf"), dtype=torch.float32, device=q.device),
                     torch.zeros(B, H, T_q, dtype=torch.float32, device=q.device),
                     torch.zeros(B, H, T_q, D, dtype=torch.float32, device=q.device))
        else:
            state = tuple(t.clone() for t in state)
    lse_view = None
    if not accumulate:
        if out is None:
            out = torch.empty(B, H, T_q, D, dtype=out_dtype or q.dtype, device=q.device)
        if lse is None:
            lse = torch.empty(B, H, T_q, dtype=torch.float32, device=q.device)
        elif not lse.is_contiguous():
            # the kernel writes lse as contiguous (B, H, T_q); a strided
            # view (e.g. one slice of a whole prompt's lse) is filled after
            lse_view, lse = lse, torch.empty(B, H, T_q, dtype=torch.float32, device=q.device)
    lib = L.lib()
    for gi, grp in enumerate(groups):
        last = gi == len(groups) - 1
        prob = L.PrefillProblem()
        prob.B, prob.H, prob.H_kv, prob.T_q, prob.D = B, H, H_kv, T_q, D
        prob.dtype = L.halo_dtype(q.dtype)
        prob.q = q.data_ptr()
        prob.q_stride_b, prob.q_stride_h, prob.q_stride_t = q.stride(0), q.stride(1), q.stride(2)
        prob.q_pos0 = int(query_pos_offset)
        prob.scale = float(scale)
        if events is not None and last:
            prob.event_begin, prob.event_end = events
        structs, keep = [], []
        for (k, v, start, causal) in grp:
            _require_cuda(k, "k")
            st, t = make_chunk(k, v, start, causal)
            structs.append(st)
            keep.append(t)
        arr = (L.KVChunk * max(len(structs), 1))(*structs)
        po = L.PrefillOut()
        if state is not None:
            m, l, o = state
            po.m, po.l, po.o = m.data_ptr(), l.data_ptr(), o.data_ptr()
        if accumulate or not last:
            po.mode = L.MERGE_ACCUMULATE
        else:
            po.mode = L.MERGE_FINALIZE
            po.out_dtype = L.halo_dtype(out.dtype)
            po.out = out.data_ptr()
            po.out_stride_b, po.out_stride_h, po.out_stride_t = out.stride(0), out.stride(1), \
                out.stride(2)
            po.lse = lse.data_ptr()
        with torch.cuda.device(q.device):
            need = lib.halo_prefill_workspace_bytes(ctypes.byref(prob), arr, len(structs))
            if need < 0:
                L.check(int(need), "halo_prefill_workspace_bytes")
            ws = PREFILL_WORKSPACES.get(q.device, int(need)) if need > 0 else None
            rc = lib.halo_prefill_attention_ws(ctypes.byref(prob), arr, len(structs),
                                               ctypes.byref(po),
                                               ws.data_ptr() if ws is not None else None,
                                               ws.numel() if ws is not None else 0,
                                               L.stream_handle(q.device))
        L.check(rc, "halo_prefill_attention_ws")
    if accumulate:
        return None
    if lse_view is not None:
        lse_view.copy_(lse)
        lse = lse_view
    return out, lse


def multi_query_attention(q: torch.Tensor, chunks: Sequence[tuple], *, scale: Optional[float] = None,
                          query_pos_offset: int, out_dtype: Optional[torch.dtype] = None):
    """``T_q > 1`` queries (a chunked-prefill slice) over causal chunks: query
    row ``i`` sits at global position ``query_pos_offset + i``
    (``halo/kv_cache_chunked.py:873-942``).  bf16/fp16 with head dim 64 or
    128 run the tensor-core prefill kernel; other shapes run each query row
    as one decode problem whose K/V batch stride is zero, so every row reuses
    the same chunk memory.  Returns ``(out (B, H, T_q, D_v), lse (B, H, T_q))``."""
    _require_cuda(q, "q")
    B, H, T_q, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if chunks and prefill_supported(q, chunks, scale):
        return prefill_attention(q, chunks, query_pos_offset=query_pos_offset, scale=scale,
                                 out_dtype=out_dtype)
    D_v = int(chunks[0][1].shape[-1]) if chunks else D
    H_kv = int(chunks[0][0].shape[1]) if chunks else H
    out = torch.empty(B, H, T_q, D_v, dtype=out_dtype or q.dtype, device=q.device)
    lse = torch.empty(B, H, T_q, dtype=torch.float32, device=q.device)
    qp = torch.arange(T_q, dtype=torch.int64, device=q.device) + int(query_pos_offset)
    for b in range(B):
        qb = q[b].transpose(0, 1).contiguous()   # (T_q, H, D)
        structs, keep = [], []
        for (k, v, start, causal) in chunks:
            s, t = make_chunk(k[b:b + 1], v[b:b + 1], start, causal, batch_stride_zero=True)
            structs.append(s)
            keep.append(t)
        ob = out[b].transpose(0, 1)          # (T_q, H, D_v) view
        lb = torch.empty(T_q, H, dtype=torch.float32, device=q.device)
        mg = L.MergeArgs()
        mg.mode = L.MERGE_FINALIZE
        mg.out_dtype = L.halo_dtype(ob.dtype)
        mg.out = ob.data_ptr()
        mg.out_stride_b, mg.out_stride_h = ob.stride(0), ob.stride(1)
        mg.lse = lb.data_ptr()
        decode_raw(qb, structs, H_kv, D_v, scale=scale, q_pos=qp, merge=mg)
        lse[b] = lb.transpose(0, 1)
    return out, lse


def multi_query_accumulate(q: torch.Tensor, chunks: Sequence[tuple], m: torch.Tensor,
                           l: torch.Tensor, o: torch.Tensor, *, scale: float,
                           query_pos_offset: int) -> None:
    """Fold ``chunks`` into running fp32 state for ``T_q > 1`` queries: query
    row ``i`` sits at position ``query_pos_offset + i``; causal chunks hide
    keys after it.  State layout ``m, l (B, T_q, H)``, ``o (B, T_q, H, D_v)``
    (contiguous), i.e. rows ordered (query row, head) per batch."""
    _require_cuda(q, "q")
    B, H, T_q, D = q.shape
    qp = torch.arange(T_q, dtype=torch.int64, device=q.device) + int(query_pos_offset)
    for b in range(B):
        table = ChunkTable(chunks, batch_stride_zero=True, batch=slice(b, b + 1))
        qb = q[b].transpose(0, 1).contiguous()          # (T_q, H, D)
        mg = L.MergeArgs()
        mg.mode = L.MERGE_ACCUMULATE
        mg.m, mg.l, mg.o = m[b].data_ptr(), l[b].data_ptr(), o[b].data_ptr()
        _decode_table(qb, table, scale=scale, q_pos=qp, merge=mg)


def lse_merge(m_parts: torch.Tensor, l_parts: Optional[torch.Tensor], o_parts: torch.Tensor, *,
              out_dtype: torch.dtype = torch.float32, out: Optional[torch.Tensor] = None,
              lse: Optional[torch.Tensor] = None, parts_major: bool = False):
    """Merge ``P`` partial states into ``(out (B, H, D_v), lse (B, H))``; the
    P-way form of ``halo/kv_cache_chunked.py:194-239``.

    Row-major (default): ``m/l (B, H, P)``, ``o (B, H, P, D_v)``.
    ``parts_major``: ``m/l (P, B, H)``, ``o (P, B, H, D_v)`` (e.g. gathered
    from P GPUs).  ``l_parts=None`` means every part is normalised (l = 1,
    ``m`` is its LSE).  All fp32.
    """
    if parts_major:
        P, B, H = m_parts.shape
    else:
        B, H, P = m_parts.shape
    D_v = o_parts.shape[-1]
    R = B * H
    for t in (m_parts, l_parts, o_parts):
        if t is None:
            continue
        _require_cuda(t, "partial")
        if t.dtype != torch.float32 or t.stride(-1) != 1:
            raise L.HaloError("partials must be fp32 with a contiguous last dim",
                              L.HALO_ERR_INVALID_ARG)
    if parts_major:
        ps, rs = m_parts.stride(0), 1
        ops_, ors = o_parts.stride(0), D_v
        if m_parts.stride(2) != 1 or m_parts.stride(1) != H or o_parts.stride(1) != H * D_v:
            raise L.HaloError("parts-major partials need contiguous (B, H) rows", L.HALO_ERR_INVALID_ARG)
    else:
        m_parts = m_parts.contiguous()
        o_parts = o_parts.contiguous()
        l_parts = l_parts.contiguous() if l_parts is not None else None
        ps, rs, ops_, ors = 1, P, D_v, P * D_v
    dev = m_parts.device
    if out is None:
        out = torch.empty(B, H, D_v, dtype=out_dtype, device=dev)
    if lse is None:
        lse = torch.empty(B, H, dtype=torch.float32, device=dev)
    mg = L.MergeArgs()
    mg.mode = L.MERGE_FINALIZE
    mg.out_dtype = L.halo_dtype(out.dtype)
    mg.out = out.data_ptr()
    mg.out_stride_b, mg.out_stride_h = out.stride(0), out.stride(1)
    mg.lse = lse.data_ptr()
    with torch.cuda.device(dev):
        rc = L.lib().halo_lse_merge(B, H, D_v, P, m_parts.data_ptr(),
                                    l_parts.data_ptr() if l_parts is not None else None,
                                    o_parts.data_ptr(), ps, rs, ops_, ors, ctypes.byref(mg),
                                    L.stream_handle(dev))
    L.check(rc, "halo_lse_merge")
    return out, lse
