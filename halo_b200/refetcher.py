"""Predictive refetcher (``halo/refetcher.py`` in lzbaclz/HALO, :24-114):
blocks predicted hot for the next ``lookahead`` steps that are not on the GPU
tier are moved up on a side CUDA stream; hits and misses are counted."""
from __future__ import annotations


class HALORefetcher:
    """Issue block moves to the GPU tier for predicted-hot blocks."""

    def __init__(self, config, *, storage) -> None:
        self.cfg = config
        self.storage = storage
        self._stream = None
        self._inflight: set = set()
        self.hits = 0
        self.misses = 0

    def predict_hot(self, *, layer: int, last_hot_indices, last_score):
        """The current hot set widened by ``lookahead`` runner-up positions
        (every position when ``hot_ratio >= 1``), sorted."""
        import torch
        K = last_score.shape[-1]
        if self.cfg.hot_ratio >= 1.0:
            return torch.arange(K, device=last_score.device, dtype=torch.long)
        k = min(max(int(self.cfg.hot_ratio * K), 1) + self.cfg.lookahead, K)
        return torch.topk(last_score, k=k).indices.sort().values

    def schedule(self, *, layer: int, predicted_indices) -> None:
        import torch
        if isinstance(predicted_indices, torch.Tensor):
            predicted_indices = predicted_indices.tolist()
        seen = set()
        for pos in predicted_indices:
            blk = int(pos) // self.cfg.block_size
            if blk in seen:
                continue
            seen.add(blk)
            where = self.storage.locate_block(layer=layer, block=blk)
            if where == "gpu":
                self.hits += 1
                continue
            if (layer, blk) in self._inflight:
                continue
            self.misses += 1
            self._inflight.add((layer, blk))
            self._issue(layer, blk, where)

    def wait(self) -> None:
        import torch
        if torch.cuda.is_available() and self._stream is not None:
            torch.cuda.current_stream().wait_stream(self._stream)
        self._inflight.clear()

    def _issue(self, layer: int, block: int, src: str) -> None:
        import torch
        if self.cfg.async_refetch and torch.cuda.is_available():
            if self._stream is None:
                self._stream = torch.cuda.Stream()
            self._stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self._stream):
                self.storage.move_block(layer=layer, block=block, src=src, dst="gpu")
        else:
            self.storage.move_block(layer=layer, block=block, src=src, dst="gpu")

    def __repr__(self) -> str:  # pragma: no cover
        tot = self.hits + self.misses
        return f"HALORefetcher(hit_rate={(self.hits / tot) if tot else 0.0:.3f}, inflight={len(self._inflight)})"


__all__ = ["HALORefetcher"]
