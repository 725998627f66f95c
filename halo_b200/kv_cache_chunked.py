"""``HALOCacheChunked``: identity-preserving tiered KV cache (Path D) on B200.

Drop-in for ``halo/kv_cache_chunked.py`` of lzbaclz/HALO (:114-996): same
constructor, ``update`` / ``compute_attention`` / ``get_seq_length`` /
``telemetry`` / ``reset`` and the private fields its tests and harnesses use
(``_mode``, ``_cold_k``, ``_cold_v``, ``_quest_scorer``, ``_last_query``,
``_peel_to_cold``, ``_iter_layer_kv``, static ``_chunk_attention`` and
``_lse_merge``).

How it runs here:

* Warm-up mode keeps the parent ``DynamicCache`` rows on the GPU (one-shot
  attention).  The first one-token update after the cache exceeds
  ``2 * chunk_size`` rows flips to chunked mode (:319-329); afterwards every
  layer keeps at most ``recent_window + chunk_size`` rows on the GPU
  (:330-334).
* Peeled rows go to a per-layer pinned host arena ``(B, H_kv, T_cap, D)``
  with one pitched DMA on a side copy stream -- no host synchronisation and
  no O(T) concatenation (the reference copies synchronously and
  ``torch.cat``s a growing host tensor, :482-521).
* ``compute_attention`` runs the split-KV kernel over the GPU-resident rows
  first, while the copy stream streams the cold rows into a double-buffered
  HBM staging ring (one pitched DMA per slot); each staged slot is folded
  into one running fp32 ``(m, l, o)`` state by the same kernel, and the last
  launch finalises ``o / l``.  The result equals the reference's chunk walk
  (``_chunk_attention`` + ``_lse_merge``) up to fp32 reduction order.
* Everything runs on CUDA; CPU tensors raise (no CPU path).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

from halo_b200.kv_cache import HALOCache


@dataclass
class _ChunkedAttentionStats:
    """Telemetry of one attention call on one layer."""

    hot_positions: int = 0
    cold_positions: int = 0
    n_chunks: int = 0
    chunk_size: int = 0
    peak_staging_bytes: int = 0
    used_lse_merge: bool = False
    dma_bytes: int = 0


class _ColdTier:
    """One layer's cold rows: pinned host arena ``(B, H_kv, T_cap, D)``."""

    def __init__(self):
        self.k = None
        self.v = None
        self.T = 0

    def reserve(self, like_k, like_v, rows: int, stream) -> None:
        import torch
        need = self.T + rows
        if self.k is not None and self.k.shape[-2] >= need:
            return
        cap = max(need, 2 * (self.k.shape[-2] if self.k is not None else 0), 1024)
        pin = torch.cuda.is_available()
        B, H = like_k.shape[0], like_k.shape[1]
        nk = torch.empty(B, H, cap, like_k.shape[-1], dtype=like_k.dtype, pin_memory=pin)
        nv = torch.empty(B, H, cap, like_v.shape[-1], dtype=like_v.dtype, pin_memory=pin)
        if self.k is not None and self.T > 0:
            if stream is not None:
                stream.synchronize()   # pending DMAs into the old arena must land first
            nk[..., :self.T, :].copy_(self.k[..., :self.T, :])
            nv[..., :self.T, :].copy_(self.v[..., :self.T, :])
        self.k, self.v = nk, nv


def _pitched(t):
    """(ptr, pitch_bytes, width_bytes, height) of a (B, H, n, D) view whose
    (B, H) rows are uniformly spaced and each row's n*D elements contiguous."""
    B, H, n, D = t.shape
    if t.stride(3) != 1 or (n > 1 and t.stride(2) != D) or (B > 1 and t.stride(0) != H * t.stride(1)):
        raise ValueError("tensor view is not 2-D pitchable")
    e = t.element_size()
    return t.data_ptr(), t.stride(1) * e, n * D * e, B * H


def _copy_rows(dst, src, stream) -> None:
    """One pitched DMA of a (B, H, n, D) view into another (any memory)."""
    from halo_b200 import _lib as L
    if src.numel() == 0:
        return
    dp, dpitch, w, h = _pitched(dst)
    sp, spitch, w2, h2 = _pitched(src)
    assert w == w2 and h == h2, "copy shape mismatch"
    L.check(L.lib().halo_copy2d_async(dp, dpitch, sp, spitch, w, h, stream.cuda_stream),
            "halo_copy2d_async")


class _ColdView:
    """Mapping-style view ``layer -> (B, H_kv, T_cold, D)`` CPU tensor of the
    cold tier (reference field ``_cold_k`` / ``_cold_v``).  Reading
    synchronises the copy stream; assigning replaces a layer's cold rows."""

    def __init__(self, cache, which: str):
        self._c, self._w = cache, which

    def _tier(self, layer):
        return self._c._cold.get(layer)

    def get(self, layer, default=None):
        t = self._tier(layer)
        if t is None or t.T == 0:
            return default
        self._c._sync_copies()
        arena = t.k if self._w == "k" else t.v
        return arena[..., :t.T, :]

    def __getitem__(self, layer):
        r = self.get(layer)
        if r is None:
            raise KeyError(layer)
        return r

    def __setitem__(self, layer, tensor) -> None:
        self._c._set_cold(layer, self._w, tensor)

    def __contains__(self, layer) -> bool:
        t = self._tier(layer)
        return t is not None and t.T > 0

    def keys(self):
        return [l for l, t in self._c._cold.items() if t.T > 0]

    def values(self):
        return [self[l] for l in self.keys()]

    def items(self):
        return [(l, self[l]) for l in self.keys()]

    def __len__(self) -> int:
        return len(self.keys())

    def __bool__(self) -> bool:
        return len(self) > 0

    def clear(self) -> None:
        self._c._cold.clear()


class HALOCacheChunked(HALOCache):
    """Tiered KV cache: cold rows in pinned host DRAM, recent rows in HBM,
    exact attention over both through split-KV decode + LSE merge."""

    #: bytes of one HBM staging slot (two slots are double-buffered)
    staging_slot_bytes: int = 64 << 20

    def __init__(self, *, config, storage, scorer, demoter, refetcher,
                 chunk_size: int = 512, recent_window: int = 64, use_triton: bool = False) -> None:
        super().__init__(config=config, storage=storage, scorer=scorer, demoter=demoter,
                         refetcher=refetcher)
        self.chunk_size = chunk_size
        self.recent_window = recent_window
        # The reference's opt-in Triton switch; the CUDA kernels are the only
        # attention path here, so the flag is kept for API compatibility.
        self.use_triton = bool(use_triton)
        self._mode = "warmup"
        self._cold: dict = {}
        self._cold_k = _ColdView(self, "k")
        self._cold_v = _ColdView(self, "v")
        self._stats: dict = {}
        self._dma_bytes_cumulative = 0
        self._quest_scorer = None
        self._last_query: dict = {}
        self._copy_streams: dict = {}
        self._staging: dict = {}

    # ------------------------------------------------------------------ reference helpers
    @staticmethod
    def _lse_merge(out_a, lse_a, out_b, lse_b):
        """Two-way LSE merge of partial results (``_lse_merge`` contract,
        ``halo/kv_cache_chunked.py:194-239``) on the GPU merge kernel:
        ``(B, H, T_q, D_v)`` outputs and ``(B, H, T_q)`` LSEs in, fp32 out."""
        import torch
        from halo_b200 import ops
        B, H, T_q, D_v = out_a.shape
        m = torch.stack([lse_a.float(), lse_b.float()], 0).permute(1, 3, 2, 0)   # (B, T_q, H, 2)
        o = torch.stack([out_a.float(), out_b.float()], 0).permute(1, 3, 2, 0, 4)  # (B, T_q, H, 2, D)
        m = m.reshape(B * T_q, H, 2).contiguous()
        o = o.reshape(B * T_q, H, 2, D_v).contiguous()
        out, lse = ops.lse_merge(m, None, o)
        return (out.view(B, T_q, H, D_v).permute(0, 2, 1, 3),
                lse.view(B, T_q, H).permute(0, 2, 1))

    @staticmethod
    def _chunk_attention(q, k_chunk, v_chunk, *, scaling: Optional[float] = None,
                         causal_mask=None):
        """Single-chunk attention ``(out, lse)`` in fp32 (``_chunk_attention``
        contract, ``halo/kv_cache_chunked.py:241-276``) on the GPU kernels.
        ``causal_mask`` is the reference's additive ``(T_q, T_c)`` mask; only
        masks of the form ``j <= offset + i`` are supported (the form
        ``compute_attention`` builds)."""
        import torch
        from halo_b200 import ops
        T_q, T_c = q.shape[-2], k_chunk.shape[-2]
        if causal_mask is None:
            if T_q == 1:
                out, lse = ops.chunked_decode(q, [(k_chunk, v_chunk, 0, False)], scale=scaling,
                                              out_dtype=torch.float32)
                return out.unsqueeze(2), lse.unsqueeze(2)
            offset = T_c   # no mask: every key visible to every query row
        else:
            allowed = torch.isfinite(causal_mask.float())
            i = torch.arange(T_q, device=allowed.device).unsqueeze(-1)
            j = torch.arange(T_c, device=allowed.device).unsqueeze(0)
            rows = allowed.any(dim=-1).nonzero()
            offset = (int(allowed[rows[0, 0]].sum().item()) - 1 - int(rows[0, 0])) if rows.numel() else -T_q - 1
            if not torch.equal(allowed, j <= offset + i):
                raise NotImplementedError("only causal masks of the form j <= offset + i are supported")
        return ops.multi_query_attention(q, [(k_chunk, v_chunk, 0, True)], scale=scaling,
                                         query_pos_offset=offset, out_dtype=torch.float32)

    # ------------------------------------------------------------------ HF cache API
    def update(self, key_states, value_states, layer_idx, *args, **kwargs):
        """Append through ``DynamicCache.update``; flip warm-up -> chunked on
        the first one-token update past ``2 * chunk_size`` rows, and in chunked
        mode peel back to ``recent_window`` rows once a layer exceeds
        ``recent_window + chunk_size`` (``halo/kv_cache_chunked.py:279-336``)."""
        T_new = key_states.shape[-2]
        K, V = super().update(key_states, value_states, layer_idx, *args, **kwargs)
        if self._quest_scorer is not None and K is not None and K.numel() > 0:
            try:
                self._quest_scorer.observe_keys(layer_idx, K)
            except Exception:
                pass
        if self._mode == "warmup":
            if T_new == 1 and K is not None and K.numel() > 0 and K.shape[-2] > 2 * self.chunk_size:
                self._mode = "chunked"
                self._peel_to_cold(layer_idx)
                K, V = self._get_layer_kv(layer_idx)
        elif self._mode == "chunked":
            if K is not None and K.shape[-2] > self.recent_window + self.chunk_size:
                self._peel_to_cold(layer_idx)
                K, V = self._get_layer_kv(layer_idx)
        return K, V

    def _iter_layer_kv(self):
        """Yield ``(layer_idx, layer_obj, K, V)`` for transformers 5.x
        (``self.layers``) and the older list layout."""
        if isinstance(getattr(self, "layers", None), list):
            for i, layer in enumerate(self.layers):
                K = getattr(layer, "keys", None)
                V = getattr(layer, "values", None)
                yield i, layer, K, V
            return
        if isinstance(getattr(self, "key_cache", None), list):
            for i in range(len(self.key_cache)):
                yield i, None, self.key_cache[i], self.value_cache[i]

    def _get_layer_kv(self, layer_idx):
        for i, _, k, v in self._iter_layer_kv():
            if i == layer_idx:
                return k, v
        return None, None

    def _replace_layer_kv(self, layer_idx, new_k, new_v) -> None:
        for i, layer, _, _ in self._iter_layer_kv():
            if i != layer_idx:
                continue
            if layer is not None:
                layer.keys, layer.values = new_k, new_v
            else:
                self.key_cache[layer_idx], self.value_cache[layer_idx] = new_k, new_v
            return

    def _copy_stream(self, device):
        import torch
        s = self._copy_streams.get(device.index)
        if s is None:
            s = torch.cuda.Stream(device=device)
            self._copy_streams[device.index] = s
        return s

    def _sync_copies(self) -> None:
        for s in self._copy_streams.values():
            s.synchronize()

    def _set_cold(self, layer, which, tensor) -> None:
        """Install ``tensor`` (B, H_kv, T, D) as a layer's cold K or V rows."""
        import torch
        self._sync_copies()
        t = self._cold.setdefault(layer, _ColdTier())
        T = tensor.shape[-2]
        arena = getattr(t, which)
        if arena is None or arena.shape[-2] < T or arena.shape[:2] != tensor.shape[:2]:
            pin = torch.cuda.is_available()
            arena = torch.empty(*tensor.shape[:2], max(T, 1024), tensor.shape[-1],
                                dtype=tensor.dtype, pin_memory=pin)
            setattr(t, which, arena)
        arena[..., :T, :].copy_(tensor)
        t.T = T

    def _peel_to_cold(self, layer_idx) -> None:
        """Move all but ``recent_window`` GPU rows of a layer to the cold tier
        (``halo/kv_cache_chunked.py:384-548``): asynchronous pitched DMA into
        the pinned arena on the copy stream.  With a Quest scorer attached and
        a stashed query, the Quest-top pages plus the recent rows stay on the
        GPU and the rest are peeled (:416-457)."""
        import torch
        k_gpu, v_gpu = self._get_layer_kv(layer_idx)
        if k_gpu is None or k_gpu.numel() == 0:
            return
        T = k_gpu.shape[-2]
        recent = min(self.recent_window, T)
        peel = T - recent
        if peel <= 0:
            return
        keep_idx = None
        q_last = self._last_query.get(layer_idx) if self._quest_scorer is not None else None
        if q_last is not None:
            try:
                hot_pages = self._quest_scorer.select_hot_pages(layer_idx, q_last)
            except Exception:
                hot_pages = None
            if hot_pages is not None and hot_pages.numel() > 0:
                p = self._quest_scorer.page_size
                keep = torch.zeros(T, dtype=torch.bool)
                for pg in hot_pages.tolist():
                    if pg * p < T:
                        keep[pg * p:min(pg * p + p, T)] = True
                if recent > 0:
                    keep[-recent:] = True
                n_keep = int(keep.sum())
                if 0 < n_keep < T:
                    keep_idx = keep.nonzero().squeeze(-1).to(k_gpu.device)
                    peel_idx = (~keep).nonzero().squeeze(-1).to(k_gpu.device)
                    peel = int(peel_idx.numel())
        if not k_gpu.is_cuda:
            raise RuntimeError("HALOCacheChunked needs CUDA tensors (no CPU path)")
        dev = k_gpu.device
        cs = self._copy_stream(dev)
        cur = torch.cuda.current_stream(dev)
        if keep_idx is not None:
            src_k = k_gpu.index_select(-2, peel_idx)
            src_v = v_gpu.index_select(-2, peel_idx)
            new_k = k_gpu.index_select(-2, keep_idx)
            new_v = v_gpu.index_select(-2, keep_idx)
        else:
            src_k, src_v = k_gpu[..., :peel, :], v_gpu[..., :peel, :]
            new_k = k_gpu[..., peel:, :].contiguous()
            new_v = v_gpu[..., peel:, :].contiguous()
        tier = self._cold.setdefault(layer_idx, _ColdTier())
        tier.reserve(src_k, src_v, peel, cs)
        cs.wait_stream(cur)
        _copy_rows(tier.k[..., tier.T:tier.T + peel, :], src_k, cs)
        _copy_rows(tier.v[..., tier.T:tier.T + peel, :], src_v, cs)
        for t in (k_gpu, v_gpu, src_k, src_v):
            t.record_stream(cs)   # keep GPU memory alive until the DMA ran
        tier.T += peel
        self._replace_layer_kv(layer_idx, new_k, new_v)
        self._dma_bytes_cumulative += int(src_k.element_size() * (src_k.numel() + src_v.numel()))
        # Demotion bookkeeping in block_size units (the rows themselves
        # already live in the cold arena).
        block = max(1, getattr(self.cfg, "block_size", 32))
        self.demoted_blocks_total += (peel + block - 1) // block

    def get_seq_length(self, layer_idx: int = 0) -> int:
        """Cold + GPU rows: the true position count (RoPE positions)."""
        t = self._cold.get(layer_idx)
        cold = t.T if t is not None else 0
        try:
            gpu = super().get_seq_length(layer_idx)
        except Exception:
            gpu = 0
        return cold + gpu

    def get_max_cache_shape(self):
        return None

    # ------------------------------------------------------------------ attention
    def _staging_buffers(self, dev, B, H_kv, D, Dv, dtype, rows):
        import torch
        key = (dev.index, B, H_kv, D, Dv, dtype, rows)
        st = self._staging.get(key)
        if st is None:
            mk = lambda d: torch.empty(B, H_kv, rows, d, dtype=dtype, device=dev)
            st = {"k": [mk(D), mk(D)], "v": [mk(Dv), mk(Dv)],
                  "ready": [torch.cuda.Event(), torch.cuda.Event()],
                  "free": [torch.cuda.Event(), torch.cuda.Event()]}
            self._staging = {key: st}   # keep one staging ring
        return st

    def compute_attention(self, q, *, layer_idx: int, scaling: Optional[float] = None,
                          query_pos_offset: Optional[int] = None):
        """Exact attention of ``q (B, H, T_q, D)`` over this layer's cold and
        GPU rows (``halo/kv_cache_chunked.py:765-964``).  Cold rows sit at
        positions ``[0, T_cold)``, GPU rows at ``T_cold + i``; causal masks
        ``key <= query_pos_offset + i`` apply only when ``T_q > 1``, with
        ``query_pos_offset`` defaulting to ``T_total - T_q``.  Returns
        ``(B, H, T_q, D_v)`` in ``q.dtype``."""
        import torch
        from halo_b200 import ops
        if self._quest_scorer is not None:
            self._last_query[layer_idx] = q.detach()
        B, H, T_q, D = q.shape
        dev = q.device
        tier = self._cold.get(layer_idx)
        T_cold = tier.T if tier is not None else 0
        gpu_k, gpu_v = self._get_layer_kv(layer_idx)
        T_gpu = gpu_k.shape[-2] if (gpu_k is not None and gpu_k.numel() > 0) else 0
        T_total = T_cold + T_gpu
        if T_total == 0:
            return torch.zeros(B, H, T_q, D, dtype=q.dtype, device=dev)
        if dev.type != "cuda":
            raise RuntimeError("HALOCacheChunked.compute_attention needs CUDA tensors (no CPU path)")
        if query_pos_offset is None:
            query_pos_offset = T_total - T_q
        scale = float(scaling) if scaling is not None else 1.0 / math.sqrt(D)
        cs_ = max(1, self.chunk_size)
        causal = T_q > 1
        last_visible = query_pos_offset + T_q - 1
        like = gpu_k if T_gpu > 0 else tier.k
        D_v = (gpu_v if T_gpu > 0 else tier.v).shape[-1]
        H_kv = like.shape[1]

        # reference telemetry: chunk count of its cold/recent walk
        def n_walk(T_part, off):
            return sum(1 for c0 in range(0, T_part, cs_) if not (causal and off + c0 > last_visible))
        n_chunks = n_walk(T_cold, 0) + n_walk(T_gpu, T_cold)

        # T_q > 1 in bf16/fp16 with head dim 64/128: tensor-core prefill kernel,
        # running state (B, H, T_q); otherwise the split-KV kernel, state in
        # (B, T_q, H) row order.
        use_pf = causal and ops.prefill_supported(q, [(like, (gpu_v if T_gpu > 0 else tier.v),
                                                        0, True)], scale)
        if use_pf:
            m = torch.full((B, H, T_q), float("-inf"), dtype=torch.float32, device=dev)
            l = torch.zeros(B, H, T_q, dtype=torch.float32, device=dev)
            o = torch.zeros(B, H, T_q, D_v, dtype=torch.float32, device=dev)
        else:
            m = torch.full((B, T_q, H), float("-inf"), dtype=torch.float32, device=dev)
            l = torch.zeros(B, T_q, H, dtype=torch.float32, device=dev)
            o = torch.zeros(B, T_q, H, D_v, dtype=torch.float32, device=dev)

        def fold(k, v, start):
            if T_q == 1:
                ops.accumulate_decode(q, [(k, v, start, False)], m.view(B, H), l.view(B, H),
                                      o.view(B, H, D_v), scale=scale, q_pos=None)
            elif use_pf:
                ops.prefill_attention(q, [(k, v, start, True)], query_pos_offset=query_pos_offset,
                                      scale=scale, state=(m, l, o), accumulate=True)
            else:
                ops.multi_query_accumulate(q, [(k, v, start, True)], m, l, o, scale=scale,
                                           query_pos_offset=query_pos_offset)

        if T_gpu > 0 and not (causal and T_cold > last_visible):
            fold(gpu_k, gpu_v, T_cold)

        dma = 0
        peak_stage = 0
        if T_cold > 0:
            cold_rows = min(T_cold, last_visible + 1) if causal else T_cold
            row_bytes = B * H_kv * (D + D_v) * like.element_size()
            slot_rows = max(cs_, (self.staging_slot_bytes // max(row_bytes, 1)) // cs_ * cs_)
            slot_rows = min(slot_rows, max(cs_, -(-cold_rows // cs_) * cs_))
            st = self._staging_buffers(dev, B, H_kv, D, D_v, like.dtype, slot_rows)
            cstream = self._copy_stream(dev)
            cur = torch.cuda.current_stream(dev)
            cstream.wait_stream(cur)   # staging memory is ordered on the compute stream
            for i, a in enumerate(range(0, cold_rows, slot_rows)):
                n = min(slot_rows, cold_rows - a)
                s = i % 2
                with torch.cuda.stream(cstream):
                    if i >= 2:
                        cstream.wait_event(st["free"][s])
                    _copy_rows(st["k"][s][..., :n, :], tier.k[..., a:a + n, :], cstream)
                    _copy_rows(st["v"][s][..., :n, :], tier.v[..., a:a + n, :], cstream)
                    st["ready"][s].record(cstream)
                cur.wait_event(st["ready"][s])
                fold(st["k"][s][..., :n, :], st["v"][s][..., :n, :], a)
                st["free"][s].record(cur)
                dma += n * row_bytes
                peak_stage = max(peak_stage, n * row_bytes)

        if use_pf:
            # no chunks: the kernel only normalises the carried state
            out, _ = ops.prefill_attention(q, [], query_pos_offset=query_pos_offset, scale=scale,
                                           state=(m, l, o), out_dtype=q.dtype)
        else:
            out = torch.where(l.unsqueeze(-1) > 0, o / l.clamp_min(1e-30).unsqueeze(-1),
                              torch.zeros_like(o)).permute(0, 2, 1, 3)
        self._stats[layer_idx] = _ChunkedAttentionStats(
            hot_positions=T_gpu, cold_positions=T_cold, n_chunks=n_chunks, chunk_size=cs_,
            peak_staging_bytes=peak_stage, used_lse_merge=n_chunks > 1, dma_bytes=dma)
        self._dma_bytes_cumulative += dma
        block = max(1, getattr(self.cfg, "block_size", 32))
        refetched = sum(max(1, (min(cs_, T_cold - c0) + block - 1) // block)
                        for c0 in range(0, T_cold, cs_)
                        if not (causal and c0 > last_visible))
        self.refetched_blocks_total += refetched
        try:
            self.refetcher.hits += refetched
        except Exception:
            pass
        return out.to(q.dtype)

    # ------------------------------------------------------------------ bookkeeping
    def telemetry(self) -> dict:
        base = super().telemetry()
        base["mode"] = self._mode
        base["dma_bytes_cumulative"] = int(self._dma_bytes_cumulative)
        if self._stats:
            st = self._stats.values()
            base["chunked_n_layers_called"] = len(self._stats)
            base["chunked_total_chunks"] = sum(s.n_chunks for s in st)
            base["chunked_peak_staging_bytes_max"] = max(s.peak_staging_bytes for s in st)
            base["chunked_used_lse_merge_any"] = any(s.used_lse_merge for s in st)
            base["chunked_total_dma_bytes"] = sum(s.dma_bytes for s in st)
        cold = [t.T for t in self._cold.values() if t.T > 0]
        if cold:
            base["cold_positions_per_layer_max"] = max(cold)
            base["cold_layers"] = len(cold)
        return base

    def reset(self) -> None:
        self._sync_copies()
        super().reset()
        self._mode = "warmup"
        self._cold.clear()
        self._stats.clear()
        self._dma_bytes_cumulative = 0
        self._last_query.clear()


__all__ = ["HALOCacheChunked"]
