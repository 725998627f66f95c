"""Placement-scorer ablations under Path D, on the B200 kernels.

Mirrors ``baselines/scorer_ablations.py`` of lzbaclz/HALO (:52-455):
``AblationScorerConfig``, the shared bookkeeping of ``_BaseAblationAdapter``
(full pages per layer, hot-page budget, counters), the four scorers and
``wrap_with_path_d_ablation_scorer``.  The selection rules are the
reference's:

* ``UniformRandomScorerAdapter`` / ``FIFOScorerAdapter`` are host-side index
  rules (a seeded CPU permutation, the most recent pages) exactly as there.
* ``HALOPressScorerAdapter`` keeps per-page mean keys in HBM
  (``halo_page_mean``, appended as pages fill) and scores
  ``alpha * attn + beta * recency + gamma * sink`` with its top-k in
  ``halo_page_press_topk`` (attention proxy ``q_g . K_mean``, min-max
  normalised, :220-268).
* ``MagicPIGSampledScorerAdapter`` takes the Quest per-page bounds from
  ``halo_page_score_topk`` and samples pages without replacement in
  proportion to ``softmax(s / temperature)`` with the reference's seeded CPU
  generator (:318-398).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from halo_b200 import _lib as L


@dataclass
class AblationScorerConfig:
    """Configuration of a Path D placement-scorer ablation cell (defaults as
    the reference)."""

    scorer_name: str = "uniform_random"
    page_size: int = 16
    memory_ratio: float = 4.0
    min_pages_selected: int = 4
    chunk_size: int = 512
    recent_window: int = 64
    use_triton: bool = True
    seed: int = 0
    halopress_alpha: float = 1.0
    halopress_beta: float = 0.5
    halopress_gamma: float = 2.0
    halopress_sink_tokens: int = 4
    halopress_refresh_window: int = 64


class _BaseAblationAdapter:
    """Full pages per layer, the hot-page budget and the counters shared by
    every scorer (the interface of ``_QuestScorerAdapter``)."""

    def __init__(self, cfg: AblationScorerConfig) -> None:
        self.cfg = cfg
        self.page_size = cfg.page_size
        self.memory_ratio = cfg.memory_ratio
        self.min_pages_selected = cfg.min_pages_selected
        self._num_full_pages: dict = {}
        self.observe_calls = 0
        self.score_calls = 0
        self.last_hot_pages_per_layer: dict = {}
        self.cumulative_hot_pages = 0

    def observe_keys(self, layer_idx: int, K_full) -> None:
        if K_full is None or K_full.numel() == 0:
            return
        n_full = K_full.shape[-2] // self.page_size
        if n_full > int(self._num_full_pages.get(layer_idx, 0)):
            self._num_full_pages[layer_idx] = n_full
        self.observe_calls += 1

    def _num_hot_pages(self, P: int) -> int:
        K = max(self.min_pages_selected, int((P + self.memory_ratio - 1) // self.memory_ratio))
        return min(K, P)

    def _record(self, layer_idx: int, topk: torch.Tensor) -> None:
        self.last_hot_pages_per_layer[layer_idx] = topk
        self.cumulative_hot_pages += int(topk.numel())
        self.score_calls += 1


class UniformRandomScorerAdapter(_BaseAblationAdapter):
    """``K`` pages uniformly at random, from a CPU generator seeded with
    ``seed + layer * 10007 + score_calls`` (reproducible)."""

    def select_hot_pages(self, layer_idx: int, query) -> Optional[torch.Tensor]:
        P = int(self._num_full_pages.get(layer_idx, 0))
        if P == 0:
            return None
        K = self._num_hot_pages(P)
        g = torch.Generator(device="cpu")
        g.manual_seed(int(self.cfg.seed) + int(layer_idx) * 10_007 + int(self.score_calls))
        topk = torch.randperm(P, generator=g)[:K].sort().values
        self._record(layer_idx, topk)
        return topk


class FIFOScorerAdapter(_BaseAblationAdapter):
    """The most recent ``K`` pages (oldest-first eviction)."""

    def select_hot_pages(self, layer_idx: int, query) -> Optional[torch.Tensor]:
        P = int(self._num_full_pages.get(layer_idx, 0))
        if P == 0:
            return None
        K = self._num_hot_pages(P)
        topk = torch.arange(P - K, P, dtype=torch.long)
        self._record(layer_idx, topk)
        return topk


def _grow(buf: Optional[torch.Tensor], shape, dtype, device, keep: int) -> torch.Tensor:
    """A (B, H_kv, cap, D) page buffer with at least shape[2] pages, keeping
    the first ``keep`` pages of ``buf``."""
    B, H_kv, need, D = shape
    if buf is not None and buf.shape[2] >= need and buf.shape[:2] == (B, H_kv):
        return buf
    cap = max(need, 2 * (buf.shape[2] if buf is not None else 0), 16)
    out = torch.empty(B, H_kv, cap, D, dtype=dtype, device=device)
    if buf is not None and keep > 0:
        out[:, :, :keep].copy_(buf[:, :, :keep])
    return out


class HALOPressScorerAdapter(_BaseAblationAdapter):
    """Closed-form ``alpha * attn + beta * recency + gamma * sink`` page
    scorer with the attention proxy ``q . K_mean`` over per-page mean keys."""

    def __init__(self, cfg: AblationScorerConfig) -> None:
        super().__init__(cfg)
        self._kmean_buf: dict = {}
        self._k_mean: dict = {}
        self._pages_meaned: dict = {}

    def observe_keys(self, layer_idx: int, K_full) -> None:
        super().observe_keys(layer_idx, K_full)
        if K_full is None or K_full.numel() == 0:
            return
        if not K_full.is_cuda:
            raise L.HaloError("observe_keys needs a CUDA tensor (no CPU path)",
                              L.HALO_ERR_INVALID_ARG)
        B, H_kv, T, D = K_full.shape
        n_full = T // self.page_size
        prev = int(self._pages_meaned.get(layer_idx, 0))
        if n_full <= prev:
            return
        K = K_full if K_full.stride(-1) == 1 else K_full.contiguous()
        buf = _grow(self._kmean_buf.get(layer_idx), (B, H_kv, n_full, D), K.dtype, K.device, prev)
        self._kmean_buf[layer_idx] = buf
        with torch.cuda.device(K.device):
            rc = L.lib().halo_page_mean(
                K.data_ptr(), K.stride(0), K.stride(1), K.stride(2), B, H_kv, D,
                L.halo_dtype(K.dtype), self.page_size, prev, n_full - prev, buf.data_ptr(),
                buf.stride(0), buf.stride(1), buf.stride(2), L.stream_handle(K.device))
        L.check(rc, "halo_page_mean")
        self._k_mean[layer_idx] = buf[:, :, :n_full]
        self._pages_meaned[layer_idx] = n_full

    def select_hot_pages(self, layer_idx: int, query) -> Optional[torch.Tensor]:
        if layer_idx not in self._k_mean:
            return None
        km = self._k_mean[layer_idx]
        B, H_kv, P, D = km.shape
        q = query if query.stride(-1) == 1 else query.contiguous()
        _, H, T_q, _ = q.shape
        if H % H_kv:
            raise L.HaloError("GQA mismatch", L.HALO_ERR_INVALID_ARG)
        K = self._num_hot_pages(P)
        c = self.cfg
        n_sink = min(c.halopress_sink_tokens // max(self.page_size, 1) + 1, P)
        scores = torch.empty(B, H_kv, T_q, P, dtype=torch.float32, device=q.device)
        topk = torch.empty(max(K, 1), dtype=torch.int64, device=q.device)
        with torch.cuda.device(q.device):
            rc = L.lib().halo_page_press_topk(
                q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), B, H, T_q, H_kv, D,
                L.halo_dtype(q.dtype), km.data_ptr(), km.stride(0), km.stride(1), km.stride(2),
                P, float(c.halopress_alpha), float(c.halopress_beta), float(c.halopress_gamma),
                int(c.halopress_refresh_window), int(n_sink), scores.data_ptr(), K, None,
                topk.data_ptr(), L.stream_handle(q.device))
        L.check(rc, "halo_page_press_topk")
        top = topk[:K].cpu().sort().values
        self._record(layer_idx, top)
        return top


class MagicPIGSampledScorerAdapter(_BaseAblationAdapter):
    """Pages sampled without replacement in proportion to
    ``softmax(quest_bound / temperature)`` (MagicPIG-style importance
    sampling), with a seeded CPU generator."""

    def __init__(self, cfg: AblationScorerConfig, temperature: float = 1.0) -> None:
        super().__init__(cfg)
        self.temperature = temperature
        from halo_b200.baselines.quest_path_d import QuestPathDConfig, _QuestScorerAdapter
        self._quest = _QuestScorerAdapter(QuestPathDConfig(
            page_size=cfg.page_size, memory_ratio=cfg.memory_ratio,
            min_pages_selected=cfg.min_pages_selected))

    def observe_keys(self, layer_idx: int, K_full) -> None:
        super().observe_keys(layer_idx, K_full)
        self._quest.observe_keys(layer_idx, K_full)

    def select_hot_pages(self, layer_idx: int, query) -> Optional[torch.Tensor]:
        if layer_idx not in self._quest._k_min:
            return None
        P = self._quest._k_min[layer_idx].shape[2]
        _, _, per_page = self._quest._run(layer_idx, query, 0, per_page_only=True)
        K = self._num_hot_pages(P)
        probs = torch.softmax(per_page / max(self.temperature, 1e-6), dim=0)
        g = torch.Generator(device="cpu")
        g.manual_seed(int(self.cfg.seed) + int(layer_idx) * 10_007 + int(self.score_calls) + 9001)
        topk = torch.multinomial(probs.cpu(), num_samples=K, replacement=False,
                                 generator=g).sort().values
        self._record(layer_idx, topk)
        return topk


_SCORER_REGISTRY = {
    "uniform_random": UniformRandomScorerAdapter,
    "halopress": HALOPressScorerAdapter,
    "fifo": FIFOScorerAdapter,
    "magicpig_sampled": MagicPIGSampledScorerAdapter,
}


def wrap_with_path_d_ablation_scorer(model, cfg: AblationScorerConfig):
    """Install Path D with the scorer named by ``cfg.scorer_name`` (``"quest"``
    goes through ``wrap_with_quest_path_d``); the cache's ``_quest_scorer``
    slot holds the adapter, as in the reference (:400-446)."""
    if cfg.scorer_name == "quest":
        from halo_b200.baselines.quest_path_d import QuestPathDConfig, wrap_with_quest_path_d
        return wrap_with_quest_path_d(model, QuestPathDConfig(
            page_size=cfg.page_size, memory_ratio=cfg.memory_ratio,
            min_pages_selected=cfg.min_pages_selected, chunk_size=cfg.chunk_size,
            recent_window=cfg.recent_window, use_triton=cfg.use_triton))
    if cfg.scorer_name not in _SCORER_REGISTRY:
        raise ValueError(f"unknown scorer_name={cfg.scorer_name!r}; "
                         f"expected one of {sorted(set(_SCORER_REGISTRY) | {'quest'})}")
    from halo_b200.policy import HALOConfig, wrap_with_halo
    wrap_with_halo(model, HALOConfig(chunked=True, chunk_size=cfg.chunk_size,
                                     recent_window=cfg.recent_window,
                                     hot_ratio=1.0 / max(1.0, cfg.memory_ratio),
                                     use_triton=cfg.use_triton))
    model._halo_cache._quest_scorer = _SCORER_REGISTRY[cfg.scorer_name](cfg)
    model._ablation_scorer_cfg = cfg
    return model


__all__ = ["AblationScorerConfig", "UniformRandomScorerAdapter", "HALOPressScorerAdapter",
           "FIFOScorerAdapter", "MagicPIGSampledScorerAdapter", "wrap_with_path_d_ablation_scorer"]
