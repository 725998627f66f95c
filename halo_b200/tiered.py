"""Scorer-driven tiered decode: hot chunks in HBM, cold chunks in pinned host
DRAM, the top-k cold chunks by Quest score refetched on a side stream.

This is the decode step of HALO's tiered configuration (lzbaclz/HALO:
``baselines/quest_path_d.py:153-205`` picks pages, ``halo/refetcher.py:24-114``
and ``halo/memory_tier.py:181-258`` move blocks between the DRAM and GPU
tiers, ``halo/kv_cache_chunked.py:571-964`` attends chunk by chunk), built as
one pipeline per layer:

1. page scores + top-k over the cold chunks (``halo_page_score_topk``; hot
   chunks are excluded), indices copied to a pinned host buffer;
2. attention over the hot chunks starts at once on the compute stream
   (split-KV kernel, normalised ``(out, lse)`` kept as fp32 state);
3. when the indices land, the chunks not already resident in the layer's
   GPU slot cache are copied from the pinned arena into free slots with one
   pitched DMA per tensor (``halo_copy2d_async``) on the copy stream (delta
   refetch; least recently selected slots are reused first);
4. the compute stream waits for those copies and folds the selected chunks
   into the hot state (one more split-KV launch + merge).
"""
from __future__ import annotations

import ctypes
import math
from collections import OrderedDict
from typing import Optional, Sequence

import torch

from halo_b200 import _lib as L
from halo_b200 import ops


class TieredLayer:
    """One layer's KV split into hot (HBM) and cold (pinned host) chunks.

    ``k, v``: the layer's full ``(B, H_kv, T, D)`` rows on the GPU, used once
    to build the tiers (summaries of every chunk, the hot rows, the pinned
    cold arena).  ``hot_chunks``: chunk indices kept in HBM.  ``n_slots``:
    GPU slots for refetched cold chunks (at least the number selected per
    step).  Chunk ``c`` holds rows ``[c*chunk, (c+1)*chunk)`` at those global
    positions.
    """

    def __init__(self, k: torch.Tensor, v: torch.Tensor, *, chunk_size: int,
                 hot_chunks: Sequence[int], n_slots: int, copy_stream=None):
        if not (k.is_cuda and v.is_cuda):
            raise L.HaloError("TieredLayer needs CUDA tensors (no CPU path)", L.HALO_ERR_INVALID_ARG)
        B, H_kv, T, D = k.shape
        if T % chunk_size:
            raise L.HaloError("context must be whole chunks", L.HALO_ERR_INVALID_ARG)
        self.B, self.H_kv, self.D, self.C = B, H_kv, D, chunk_size
        self.dev = k.device
        self.dtype = k.dtype
        self.P = T // chunk_size
        self.hot = sorted(int(c) for c in hot_chunks)
        self.cold = [c for c in range(self.P) if c not in set(self.hot)]
        self._cold_pos = {c: i for i, c in enumerate(self.cold)}
        C = chunk_size
        k = k.contiguous()
        v = v.contiguous()
        # chunk summaries (page = chunk), exact min/max in the key dtype
        self.kmin = torch.empty(B, H_kv, self.P, D, dtype=k.dtype, device=self.dev)
        self.kmax = torch.empty_like(self.kmin)
        with torch.cuda.device(self.dev):
            rc = L.lib().halo_page_summary(
                k.data_ptr(), k.stride(0), k.stride(1), k.stride(2), B, H_kv, D,
                L.halo_dtype(k.dtype), C, 0, self.P, self.kmin.data_ptr(), self.kmax.data_ptr(),
                self.kmin.stride(0), self.kmin.stride(1), self.kmin.stride(2),
                L.stream_handle(self.dev))
        L.check(rc, "halo_page_summary")
        # hot rows: one compact buffer, chunk views into it
        n_hot = len(self.hot)
        self.k_hot = torch.empty(B, H_kv, n_hot * C, D, dtype=k.dtype, device=self.dev)
        self.v_hot = torch.empty_like(self.k_hot)
        for i, c in enumerate(self.hot):
            self.k_hot[:, :, i * C:(i + 1) * C].copy_(k[:, :, c * C:(c + 1) * C])
            self.v_hot[:, :, i * C:(i + 1) * C].copy_(v[:, :, c * C:(c + 1) * C])
        # cold rows: pinned host arena (B, H_kv, n_cold*C, D)
        n_cold = len(self.cold)
        self.k_cold = torch.empty(B, H_kv, n_cold * C, D, dtype=k.dtype).pin_memory()
        self.v_cold = torch.empty_like(self.k_cold).pin_memory()
        for i, c in enumerate(self.cold):
            self.k_cold[:, :, i * C:(i + 1) * C].copy_(k[:, :, c * C:(c + 1) * C])
            self.v_cold[:, :, i * C:(i + 1) * C].copy_(v[:, :, c * C:(c + 1) * C])
        torch.cuda.synchronize(self.dev)
        # GPU slots for refetched cold chunks
        self.n_slots = int(n_slots)
        self.k_slots = torch.empty(self.n_slots, B, H_kv, C, D, dtype=k.dtype, device=self.dev)
        self.v_slots = torch.empty_like(self.k_slots)
        self._slot_of: "OrderedDict[int, int]" = OrderedDict()   # chunk -> slot, LRU first
        self._free = list(range(self.n_slots))
        self.exclude = torch.zeros(self.P, dtype=torch.uint8, device=self.dev)
        self.exclude[self.hot] = 1
        self.hot_table = ops.ChunkTable([(self.k_hot[:, :, i * C:(i + 1) * C],
                                          self.v_hot[:, :, i * C:(i + 1) * C], c * C, False)
                                         for i, c in enumerate(self.hot)])
        self.copy_stream = copy_stream or torch.cuda.Stream(self.dev)
        self._idx_host = torch.empty(self.P, dtype=torch.int64).pin_memory()
        self._idx_ready = torch.cuda.Event()
        self._copied = torch.cuda.Event()
        self._ones = None
        self._scores = None
        self.stats = {"steps": 0, "selected": 0, "refetched_chunks": 0, "refetch_bytes": 0}

    @property
    def chunk_bytes(self) -> int:
        """Bytes of one chunk's K plus V."""
        return 2 * self.B * self.H_kv * self.C * self.D * self.k_hot.element_size()

    def _select(self, q3: torch.Tensor, k_sel: int) -> torch.Tensor:
        B, H, D = q3.shape
        if self._scores is None or self._scores.shape[0] != B:
            self._scores = torch.empty(B, self.H_kv, 1, self.P, dtype=torch.float32, device=self.dev)
            self._topk = torch.empty(self.P, dtype=torch.int64, device=self.dev)
            self._per_page = torch.empty(self.P, dtype=torch.float32, device=self.dev)
        with torch.cuda.device(self.dev):
            rc = L.lib().halo_page_score_topk(
                q3.data_ptr(), q3.stride(0), q3.stride(1), 0, B, H, 1, self.H_kv, D,
                L.halo_dtype(q3.dtype), self.kmin.data_ptr(), self.kmax.data_ptr(),
                self.kmin.stride(0), self.kmin.stride(1), self.kmin.stride(2), self.P,
                self._scores.data_ptr(), self.exclude.data_ptr(), k_sel,
                self._per_page.data_ptr(), self._topk.data_ptr(), L.stream_handle(self.dev))
        L.check(rc, "halo_page_score_topk")
        return self._topk[:k_sel]

    def _refetch(self, chunks: Sequence[int], copy_events: Optional[tuple] = None) -> int:
        """Copy the chunks not resident into slots (copy stream); returns how
        many were copied.  The compute stream must wait on ``self._copied``.
        ``copy_events = (begin, end)`` (``torch.cuda.Event``) are recorded
        on the copy stream around the copies."""
        need = [c for c in chunks if c not in self._slot_of]
        for c in chunks:
            if c in self._slot_of:
                self._slot_of.move_to_end(c)
        keep = set(chunks)
        cs = self.copy_stream
        cs.wait_stream(torch.cuda.current_stream(self.dev))   # slots are free on the compute stream
        if copy_events is not None:
            copy_events[0].record(cs)
        lib = L.lib()
        esz = self.k_hot.element_size()
        width = self.C * self.D * esz
        rows = self.B * self.H_kv
        src_pitch = len(self.cold) * self.C * self.D * esz
        for c in need:
            if self._free:
                s = self._free.pop()
            else:
                victim = next(x for x in self._slot_of if x not in keep)
                s = self._slot_of.pop(victim)
            self._slot_of[c] = s
            off = self._cold_pos[c] * self.C * self.D * esz
            for dst, src in ((self.k_slots[s], self.k_cold), (self.v_slots[s], self.v_cold)):
                rc = lib.halo_copy2d_async(dst.data_ptr(), width, src.data_ptr() + off, src_pitch,
                                           width, rows, ctypes.c_void_p(cs.cuda_stream))
                L.check(rc, "halo_copy2d_async")
        if copy_events is not None:
            copy_events[1].record(cs)
        self._copied.record(cs)
        return len(need)

    def step(self, q: torch.Tensor, *, k_sel: int, scale: Optional[float] = None,
             out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
             events: Optional[tuple] = None, copy_events: Optional[tuple] = None):
        """One decode query ``q (B, H, D)`` (or ``(B, H, 1, D)``): attention
        over the hot chunks and the ``k_sel`` best cold chunks.  Returns
        ``(out (B, H, D) in q.dtype, lse (B, H), selected chunk ids)``.
        ``events = (begin, end)`` bracket each split-KV launch pair (hot,
        selected) when given as two lists of raw event handles;
        ``copy_events = (begin, end)`` (``torch.cuda.Event``) bracket the
        refetch copies on the copy stream."""
        q3 = q.squeeze(2) if q.dim() == 4 else q
        q3 = q3 if q3.is_contiguous() else q3.contiguous()
        B, H, D = q3.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        cur = torch.cuda.current_stream(self.dev)
        # 1. selection, indices to the host
        top = self._select(q3, k_sel)
        self._idx_host[:k_sel].copy_(top, non_blocking=True)
        self._idx_ready.record(cur)
        # 2. hot chunks while the indices travel
        o32 = torch.empty(B, H, D, dtype=torch.float32, device=self.dev)
        lse_h = torch.empty(B, H, dtype=torch.float32, device=self.dev)
        ops.chunked_decode(q3, self.hot_table, scale=scale, out=o32, lse=lse_h,
                           events=events[0] if events else None)
        # 3. delta refetch of the selected cold chunks
        self._idx_ready.synchronize()
        chosen = [int(x) for x in self._idx_host[:k_sel].tolist()]
        n_new = self._refetch(chosen, copy_events)
        # 4. selected chunks folded into the hot state
        cur.wait_event(self._copied)
        if self._ones is None or self._ones.shape != (B, H):
            self._ones = torch.ones(B, H, dtype=torch.float32, device=self.dev)
        C = self.C
        sel = [(self.k_slots[self._slot_of[c]], self.v_slots[self._slot_of[c]], c * C, False)
               for c in chosen]
        out, lse = ops.chunked_decode(q3, sel, scale=scale, out=out, lse=lse,
                                      out_dtype=q3.dtype, prior=(lse_h, self._ones, o32),
                                      events=events[1] if events else None)
        st = self.stats
        st["steps"] += 1
        st["selected"] += len(chosen)
        st["refetched_chunks"] += n_new
        st["refetch_bytes"] += n_new * self.chunk_bytes
        return out, lse, chosen


__all__ = ["TieredLayer"]
