"""Demotion queue (``halo/demoter.py`` in lzbaclz/HALO, :20-80): blocks leave
a faster tier for a slower one, on a side CUDA stream when
``async_refetch`` is set so the hot path never waits for them."""
from __future__ import annotations

from collections import deque


class HALODemoter:
    """Queue block demotions and drain them (asynchronously on CUDA)."""

    def __init__(self, config, *, storage) -> None:
        self.cfg = config
        self.storage = storage
        self._pending: deque = deque()
        self._stream = None

    def demote(self, *, layer: int, block_indices, src: str = "gpu", dst: str = "dram") -> None:
        import torch
        if isinstance(block_indices, torch.Tensor):
            block_indices = block_indices.tolist()
        self._pending.extend((layer, int(b), src, dst) for b in block_indices)
        if self.cfg.async_refetch and torch.cuda.is_available():
            if self._stream is None:
                self._stream = torch.cuda.Stream()
            self._stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self._stream):
                self.flush()
        else:
            self.flush()

    def flush(self) -> None:
        while self._pending:
            layer, blk, src, dst = self._pending.popleft()
            self.storage.move_block(layer=layer, block=blk, src=src, dst=dst)

    def __repr__(self) -> str:  # pragma: no cover
        return f"HALODemoter(pending={len(self._pending)}, async={self.cfg.async_refetch})"


__all__ = ["HALODemoter"]
