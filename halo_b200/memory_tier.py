"""Block-addressable KV tiers (``halo/memory_tier.py`` in lzbaclz/HALO,
:31-258): a per-(layer, block) directory over lazily allocated per-tier block
buffers ``(L, max_blocks, H_kv, block, D)``.  The DRAM tier is pinned host
memory, so a block moves to or from HBM with one DMA.

The NVMe tier of the reference is outside this package's scope (it is not on
the HBM attention path); asking for it raises ``ValueError``.
"""
from __future__ import annotations

from enum import Enum
from typing import Optional


class MemoryTier(str, Enum):
    """Tier names, fast to slow."""

    GPU = "gpu"
    DRAM = "dram"
    NVME = "nvme"

    @classmethod
    def from_name(cls, name) -> "MemoryTier":
        return name if isinstance(name, cls) else cls(str(name).lower())


class TieredStorage:
    """One block buffer per tier plus a (layer, block) -> tier directory."""

    def __init__(self, *, tiers, num_layers: int, num_kv_heads: int, head_dim: int,
                 block_size: int, dtype, device, nvme_path: Optional[str] = None,
                 max_blocks: int = 4096) -> None:
        self.tiers = [MemoryTier.from_name(t) for t in tiers]
        if MemoryTier.NVME in self.tiers:
            raise ValueError("the NVMe tier is not part of halo_b200 (gpu and dram only)")
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.dtype = dtype
        self.gpu_device = device
        self.max_blocks = max_blocks
        self._shape = (num_layers, max_blocks, num_kv_heads, block_size, head_dim)
        self._directory: dict = {}
        self._buffers: dict = {}   # tier -> (keys, values), allocated on first write

    # ------------------------------------------------------------------ API
    def move_block(self, *, layer: int, block: int, src, dst) -> None:
        s, d = MemoryTier.from_name(src), MemoryTier.from_name(dst)
        if s == d:
            return
        k, v = self._block(layer, block, s)
        self._store(layer, block, k, v, d)
        self._directory[(layer, block)] = d

    def locate_block(self, *, layer: int, block: int) -> str:
        return self._directory.get((layer, block), MemoryTier.GPU).value

    def write_new_block(self, *, layer: int, block: int, keys, values, tier: str = "gpu") -> None:
        t = MemoryTier.from_name(tier)
        self._store(layer, block, keys, values, t)
        self._directory[(layer, block)] = t

    def read_block(self, *, layer: int, block: int):
        return self._block(layer, block, self._directory.get((layer, block), MemoryTier.GPU))

    # ------------------------------------------------------------------ internals
    def _ensure(self, tier: MemoryTier):
        if tier in self._buffers:
            return self._buffers[tier]
        if tier not in self.tiers:
            raise ValueError(f"Tier {tier} not requested at construction time.")
        import torch
        if tier is MemoryTier.GPU:
            kw = dict(device=self.gpu_device)
        else:
            pin = torch.cuda.is_available() and getattr(self.gpu_device, "type", "cpu") == "cuda"
            kw = dict(device="cpu", pin_memory=pin)
        bufs = (torch.empty(self._shape, dtype=self.dtype, **kw),
                torch.empty(self._shape, dtype=self.dtype, **kw))
        self._buffers[tier] = bufs
        return bufs

    def _block(self, layer, block, tier):
        k, v = self._ensure(tier)
        return k[layer, block], v[layer, block]

    def _store(self, layer, block, keys, values, tier) -> None:
        k, v = self._ensure(tier)
        k[layer, block].copy_(keys, non_blocking=True)
        v[layer, block].copy_(values, non_blocking=True)

    def __repr__(self) -> str:  # pragma: no cover
        return f"TieredStorage(tiers=[{','.join(t.value for t in self.tiers)}], blocks={self.max_blocks})"


__all__ = ["MemoryTier", "TieredStorage"]
