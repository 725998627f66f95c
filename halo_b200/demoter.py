"""Demoter: moves cooled blocks down the tier ladder (the write path of
``halo/demoter.py`` in lzbaclz/HALO, :20-80).

Requests are kept as block sets per ``(layer, src, dst)`` route; a drain
turns each route into one batched move (runs of consecutive blocks copy as
one slab, ``TieredStorage.move_blocks``).  With ``async_refetch`` the moves
run on the mover's side CUDA stream, ordered after the work already queued
on the caller's stream, so the decode path never waits for them.
"""
from __future__ import annotations

from halo_b200.memory_tier import TierMover


class HALODemoter:
    """Batched demotion of blocks between tiers."""

    def __init__(self, config, *, storage) -> None:
        self.cfg = config
        self.storage = storage
        self._routes: dict = {}              # (layer, src, dst) -> set of block ids
        self._mover = TierMover(storage, asynchronous=bool(config.async_refetch))
        self.moved_blocks = 0

    def demote(self, *, layer: int, block_indices, src: str = "gpu", dst: str = "dram") -> None:
        """Queue ``block_indices`` of ``layer`` for ``src -> dst`` and drain."""
        import torch
        ids = torch.as_tensor(block_indices, dtype=torch.long).reshape(-1).tolist()
        if ids:
            self._routes.setdefault((int(layer), src, dst), set()).update(ids)
        self.flush()

    def flush(self) -> None:
        """Issue every queued route as one batched move."""
        routes, self._routes = self._routes, {}
        for (layer, src, dst), ids in routes.items():
            self.moved_blocks += self._mover.move(layer, ids, src, dst)

    @property
    def pending(self) -> int:
        return sum(len(ids) for ids in self._routes.values())

    def __repr__(self) -> str:  # pragma: no cover
        return (f"<HALODemoter moved={self.moved_blocks} pending={self.pending} "
                f"side_stream={self._mover.asynchronous}>")


__all__ = ["HALODemoter"]
