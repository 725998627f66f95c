"""Quest + Path D: the chunk-hotness scorer on the B200 kernels.

Mirrors ``baselines/quest_path_d.py`` of lzbaclz/HALO (:42-256):
``QuestPathDConfig``, ``_QuestScorerAdapter`` (``observe_keys``,
``score_pages``, ``select_hot_pages`` and its counters) and
``wrap_with_quest_path_d``.  Page summaries, scores and top-k run in
``libhalo_sm100.so`` (``halo_page_summary`` / ``halo_page_score_topk``); the
summaries stay in HBM, appended in place.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from halo_b200 import _lib as L


@dataclass
class QuestPathDConfig:
    """Quest selection knobs + Path D chunking (defaults as the reference)."""

    page_size: int = 16
    memory_ratio: float = 4.0
    min_pages_selected: int = 4
    chunk_size: int = 512
    recent_window: int = 64
    use_triton: bool = True


class _QuestScorerAdapter:
    """Per-page K min/max summaries and Quest upper-bound selection."""

    def __init__(self, cfg: QuestPathDConfig) -> None:
        self.cfg = cfg
        self.page_size = cfg.page_size
        self.memory_ratio = cfg.memory_ratio
        self.min_pages_selected = cfg.min_pages_selected
        self._kmin_buf: dict = {}
        self._kmax_buf: dict = {}
        self._k_min: dict = {}
        self._k_max: dict = {}
        self._num_full_pages: dict = {}
        self.observe_calls = 0
        self.score_calls = 0
        self.last_hot_pages_per_layer: dict = {}
        self.cumulative_hot_pages = 0

    # ---- summaries (observe_keys, :125-150)
    def observe_keys(self, layer_idx: int, K_full) -> None:
        """Summarise pages of ``K_full (B, H_kv, T, D)`` not seen before."""
        if K_full is None or K_full.numel() == 0:
            return
        if not K_full.is_cuda:
            raise L.HaloError("observe_keys needs a CUDA tensor (no CPU path)", L.HALO_ERR_INVALID_ARG)
        B, H_kv, T, D = K_full.shape
        n_full = T // self.page_size
        prev = int(self._num_full_pages.get(layer_idx, 0))
        if n_full <= prev:
            return
        K = K_full if K_full.stride(-1) == 1 else K_full.contiguous()
        buf_min, buf_max = self._kmin_buf.get(layer_idx), self._kmax_buf.get(layer_idx)
        if buf_min is None or buf_min.shape[2] < n_full or buf_min.shape[:2] != (B, H_kv):
            cap = max(n_full, 2 * (buf_min.shape[2] if buf_min is not None else 0), 16)
            nmin = torch.empty(B, H_kv, cap, D, dtype=K.dtype, device=K.device)
            nmax = torch.empty_like(nmin)
            if buf_min is not None and prev > 0:
                nmin[:, :, :prev].copy_(buf_min[:, :, :prev])
                nmax[:, :, :prev].copy_(buf_max[:, :, :prev])
            buf_min, buf_max = nmin, nmax
            self._kmin_buf[layer_idx], self._kmax_buf[layer_idx] = buf_min, buf_max
        with torch.cuda.device(K.device):
            rc = L.lib().halo_page_summary(
                K.data_ptr(), K.stride(0), K.stride(1), K.stride(2), B, H_kv, D,
                L.halo_dtype(K.dtype), self.page_size, prev, n_full - prev, buf_min.data_ptr(),
                buf_max.data_ptr(), buf_min.stride(0), buf_min.stride(1), buf_min.stride(2),
                L.stream_handle(K.device))
        L.check(rc, "halo_page_summary")
        self._k_min[layer_idx] = buf_min[:, :, :n_full]
        self._k_max[layer_idx] = buf_max[:, :, :n_full]
        self._num_full_pages[layer_idx] = n_full
        self.observe_calls += 1

    def _run(self, layer_idx: int, query, k: int, exclude=None, per_page_only: bool = False):
        kmin, kmax = self._k_min[layer_idx], self._k_max[layer_idx]
        B, H_kv, P, D = kmin.shape
        q = query if query.stride(-1) == 1 else query.contiguous()
        Bq, H, T_q, _ = q.shape
        scores = torch.empty(B, H_kv, T_q, P, dtype=torch.float32, device=q.device)
        topk = torch.empty(max(k, 1), dtype=torch.int64, device=q.device)
        per_page = (torch.empty(P, dtype=torch.float32, device=q.device)
                    if (k > 0 or per_page_only) else None)
        ex = None
        if exclude is not None:
            ex = torch.zeros(P, dtype=torch.uint8, device=q.device)
            ex[torch.as_tensor(exclude, dtype=torch.long, device=q.device)] = 1
        with torch.cuda.device(q.device):
            rc = L.lib().halo_page_score_topk(
                q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), B, H, T_q, H_kv, D,
                L.halo_dtype(q.dtype), kmin.data_ptr(), kmax.data_ptr(), kmin.stride(0),
                kmin.stride(1), kmin.stride(2), P, scores.data_ptr(),
                ex.data_ptr() if ex is not None else None, k,
                per_page.data_ptr() if per_page is not None else None,
                topk.data_ptr() if k > 0 else None, L.stream_handle(q.device))
        L.check(rc, "halo_page_score_topk")
        return scores, (topk[:k] if k > 0 else None), per_page

    # ---- scores (score_pages, :153-181)
    def score_pages(self, layer_idx: int, query):
        """``(B, H_kv, T_q, P)`` fp32 Quest upper bounds, or ``None`` before
        any page is summarised."""
        if layer_idx not in self._k_min:
            return None
        scores, _, _ = self._run(layer_idx, query, 0)
        self.score_calls += 1
        return scores

    def num_selected(self, P: int) -> int:
        k = max(self.min_pages_selected, int((P + self.memory_ratio - 1) // self.memory_ratio))
        return min(k, P)

    # ---- top-k (select_hot_pages, :184-205)
    def select_hot_pages(self, layer_idx: int, query, *, exclude=None) -> Optional[torch.Tensor]:
        """Indices (CPU int64, best first) of the
        ``max(min_pages, ceil(P / memory_ratio))`` pages with the largest
        score max over (batch, kv-head, query); ``exclude`` lists pages that
        may not be chosen (hot chunks in the tiered decode)."""
        if layer_idx not in self._k_min:
            return None
        P = self._k_min[layer_idx].shape[2]
        k = self.num_selected(P)
        _, topk, _ = self._run(layer_idx, query, k, exclude=exclude)
        self.score_calls += 1
        top = topk.cpu()
        self.last_hot_pages_per_layer[layer_idx] = top
        self.cumulative_hot_pages += k
        return top


def wrap_with_quest_path_d(model, config: Optional[QuestPathDConfig] = None):
    """``wrap_with_halo(chunked=True)`` plus the Quest adapter on the cache
    (``baselines/quest_path_d.py:208-253``)."""
    import os
    from halo_b200 import HALOConfig, wrap_with_halo
    config = config or QuestPathDConfig()
    use_triton = config.use_triton and os.environ.get("HALO_DISABLE_TRITON", "0") != "1"
    wrap_with_halo(model, HALOConfig(chunked=True, chunk_size=config.chunk_size,
                                     recent_window=config.recent_window,
                                     hot_ratio=1.0 / max(1.0, config.memory_ratio),
                                     use_triton=use_triton))
    model._quest_path_d_config = config
    model._halo_cache._quest_scorer = _QuestScorerAdapter(config)
    return model


__all__ = ["QuestPathDConfig", "_QuestScorerAdapter", "wrap_with_quest_path_d"]
