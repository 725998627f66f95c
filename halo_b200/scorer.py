"""Closed-form per-position hotness scorer (``halo/scorer.py`` in
lzbaclz/HALO, :36-88): ``alpha * attn + beta * recency + gamma * sink``,
squashed to [0, 1], and its top-k hot set.

It drives ``HALOCache.update_hotness`` bookkeeping, not the chunked
attention; chunk-level hotness for the tiered decode is the Quest upper-bound
kernel (``halo_b200.baselines.quest_path_d``).
"""
from __future__ import annotations

from typing import TYPE_CHECKING, Optional

if TYPE_CHECKING:  # pragma: no cover
    import torch


class HALOScorer:
    """Per-position hotness from one (layer, head-mean) attention snapshot."""

    def __init__(self, config) -> None:
        self.cfg = config

    def score(self, attention: "torch.Tensor", *, step: int) -> "torch.Tensor":
        """Hotness ``(K,)`` in [0, 1] for attention mass ``(K,)`` at ``step``:
        normalised attention, recency ``exp(-(step - p)^+ / refresh_window)``
        (normalised), and a sink indicator on the first ``sink_tokens``."""
        import torch
        K = attention.shape[-1]
        dev = attention.device
        a = attention.float()
        a = a / (a.sum() + 1e-12)
        pos = torch.arange(K, device=dev, dtype=torch.float32)
        horizon = float(max(self.cfg.refresh_window, 1))
        rec = torch.exp(-(float(step) - pos).clamp(min=0.0) / horizon)
        rec = rec / (rec.sum() + 1e-12)
        sink = (pos < min(self.cfg.sink_tokens, K)).float()
        s = self.cfg.score_alpha * a + self.cfg.score_beta * rec + self.cfg.score_gamma * sink
        return s / (s.max() + 1e-12)

    def topk_hot(self, score: "torch.Tensor", *, ratio: Optional[float] = None) -> "torch.Tensor":
        """Sorted indices of the hot set: every position when ``ratio >= 1``
        (the identity case), else the top ``max(1, int(ratio * K))``."""
        import torch
        ratio = self.cfg.hot_ratio if ratio is None else ratio
        K = score.shape[-1]
        if ratio >= 1.0:
            return torch.arange(K, device=score.device, dtype=torch.long)
        k = min(max(int(ratio * K), 1), K)
        return torch.topk(score, k=k).indices.sort().values

    def jaccard(self, a: "torch.Tensor", b: "torch.Tensor") -> float:
        sa, sb = set(a.tolist()), set(b.tolist())
        if not sa and not sb:
            return 1.0
        return len(sa & sb) / max(len(sa | sb), 1)


__all__ = ["HALOScorer"]
