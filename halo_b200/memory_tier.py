"""Block-addressable KV tiers (``halo/memory_tier.py`` in lzbaclz/HALO,
:31-258): a per-(layer, block) directory over lazily allocated per-tier block
buffers ``(L, max_blocks, H_kv, block, D)``.  The DRAM tier is pinned host
memory, so a block moves to or from HBM with one DMA.

The NVMe tier (``halo/memory_tier.py:61-103, 228-258``) keeps each block as
raw bytes in two files (``keys.bin``, ``values.bin``, one slot per (layer,
block), like the reference's ``numpy.memmap`` layout, so any dtype including
bf16 round-trips bit-exactly).  The reference copies a block out of the
memory map into a new tensor; here a block is read with one positioned read
(``os.preadv``) straight into a pinned host bounce buffer.  A block bound for
HBM then crosses PCIe with a single DMA, and a block leaving HBM lands in
the bounce buffer before one positioned write.
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


class _FileTier:
    """NVMe tier: keys and values of block (layer, b) at byte offset
    ``(layer * max_blocks + b) * block_bytes`` of ``keys.bin`` / ``values.bin``
    (files sized for every slot when created).  Reads and writes go through
    a pinned host bounce buffer with one positioned syscall per tensor."""

    def __init__(self, shape, dtype, path: str, pin: bool) -> None:
        import os
        import torch
        self.shape = tuple(shape)
        self.dtype = dtype
        self.block_shape = self.shape[2:]
        itemsize = torch.tensor([], dtype=dtype).element_size()
        self.block_elems = 1
        for n in self.block_shape:
            self.block_elems *= int(n)
        self.block_bytes = self.block_elems * itemsize
        total = self.shape[0] * self.shape[1] * self.block_bytes
        os.makedirs(path, exist_ok=True)
        self.paths = (os.path.join(path, "keys.bin"), os.path.join(path, "values.bin"))
        self.fds = []
        for fp in self.paths:
            fd = os.open(fp, os.O_RDWR | os.O_CREAT, 0o644)
            os.ftruncate(fd, total)
            self.fds.append(fd)
        self.bounce = torch.empty(2, self.block_elems, dtype=dtype, pin_memory=pin)

    def _offset(self, layer: int, block: int) -> int:
        if not (0 <= layer < self.shape[0] and 0 <= block < self.shape[1]):
            raise IndexError(f"block ({layer}, {block}) outside the NVMe tier")
        return (layer * self.shape[1] + block) * self.block_bytes

    def read(self, layer: int, block: int, device=None):
        """Block ``(keys, values)`` as new tensors on ``device`` (host if None)."""
        import os
        import torch
        off = self._offset(layer, block)
        out = []
        for i, fd in enumerate(self.fds):
            view = memoryview(self.bounce[i].view(torch.uint8).numpy())
            n = os.preadv(fd, [view], off)
            if n != self.block_bytes:
                raise IOError(f"short read from {self.paths[i]} ({n} of {self.block_bytes} bytes)")
            t = self.bounce[i].view(self.block_shape)
            out.append(t.to(device, copy=True) if device is not None else t.clone())
        return out[0], out[1]

    def write(self, layer: int, block: int, keys, values) -> None:
        import os
        import torch
        off = self._offset(layer, block)
        for i, (fd, src) in enumerate(zip(self.fds, (keys, values))):
            self.bounce[i].view(self.block_shape).copy_(src)      # D2H or host copy
            if src.is_cuda:
                torch.cuda.current_stream(src.device).synchronize()
            view = memoryview(self.bounce[i].view(torch.uint8).numpy())
            n = os.pwritev(fd, [view], off)
            if n != self.block_bytes:
                raise IOError(f"short write to {self.paths[i]} ({n} of {self.block_bytes} bytes)")

    def close(self) -> None:
        import os
        for fd in self.fds:
            os.close(fd)
        self.fds = []


class TieredStorage:
    """One block buffer per tier plus a (layer, block) -> tier directory."""

    def __init__(self, *, tiers, num_layers: int, num_kv_heads: int, head_dim: int,
                 block_size: int, dtype, device, nvme_path: Optional[str] = None,
                 max_blocks: int = 4096) -> None:
        self.tiers = [MemoryTier.from_name(t) for t in tiers]
        self._nvme_path = nvme_path
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

    def locate_blocks(self, *, layer: int, blocks) -> list:
        """Tier names of several blocks of one layer, in order."""
        d = self._directory
        return [d.get((layer, int(b)), MemoryTier.GPU).value for b in blocks]

    def move_blocks(self, *, layer: int, blocks, src, dst) -> int:
        """Move several blocks of one layer between two tiers; returns how
        many moved.  Block ids are deduplicated and sorted, and each run of
        consecutive ids is one slab of the tier buffers
        ``(L, max_blocks, H_kv, block, D)``, so it moves with one copy per
        tensor (one DMA when one side is HBM and the other pinned host
        memory); the NVMe tier still moves block by block."""
        s, d = MemoryTier.from_name(src), MemoryTier.from_name(dst)
        ids = sorted({int(b) for b in blocks})
        if not ids or s == d:
            return 0
        sb, db = self._ensure(s), self._ensure(d)
        if isinstance(sb, _FileTier) or isinstance(db, _FileTier):
            for b in ids:
                self.move_block(layer=layer, block=b, src=s, dst=d)
            return len(ids)
        lo = 0
        while lo < len(ids):
            hi = lo
            while hi + 1 < len(ids) and ids[hi + 1] == ids[hi] + 1:
                hi += 1
            a, z = ids[lo], ids[hi] + 1
            for src_t, dst_t in zip(sb, db):
                dst_t[layer, a:z].copy_(src_t[layer, a:z], non_blocking=True)
            lo = hi + 1
        for b in ids:
            self._directory[(layer, b)] = d
        return len(ids)

    def write_new_block(self, *, layer: int, block: int, keys, values, tier: str = "gpu") -> None:
        t = MemoryTier.from_name(tier)
        self._store(layer, block, keys, values, t)
        self._directory[(layer, block)] = t

    def read_block(self, *, layer: int, block: int):
        return self._block(layer, block, self._directory.get((layer, block), MemoryTier.GPU))

    # ------------------------------------------------------------------ internals
    def _pin(self) -> bool:
        import torch
        return torch.cuda.is_available() and getattr(self.gpu_device, "type", "cpu") == "cuda"

    def _ensure(self, tier: MemoryTier):
        if tier in self._buffers:
            return self._buffers[tier]
        if tier not in self.tiers:
            raise ValueError(f"Tier {tier} not requested at construction time.")
        import torch
        if tier is MemoryTier.NVME:
            import os
            import tempfile
            path = (self._nvme_path or os.environ.get("HALO_NVME_PATH")
                    or os.path.join(tempfile.gettempdir(), "halo_nvme"))
            self._buffers[tier] = _FileTier(self._shape, self.dtype, path, self._pin())
            return self._buffers[tier]
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
        buf = self._ensure(tier)
        if isinstance(buf, _FileTier):
            return buf.read(layer, block)
        k, v = buf
        return k[layer, block], v[layer, block]

    def _store(self, layer, block, keys, values, tier) -> None:
        buf = self._ensure(tier)
        if isinstance(buf, _FileTier):
            buf.write(layer, block, keys, values)
            return
        k, v = buf
        k[layer, block].copy_(keys, non_blocking=True)
        v[layer, block].copy_(values, non_blocking=True)

    def refetch_block(self, *, layer: int, block: int, device):
        """The block's ``(keys, values)`` on ``device`` wherever it lives: an
        NVMe block is read into the pinned bounce buffer and crosses PCIe in
        one DMA per tensor."""
        tier = self._directory.get((layer, block), MemoryTier.GPU)
        buf = self._ensure(tier)
        if isinstance(buf, _FileTier):
            return buf.read(layer, block, device=device)
        k, v = self._block(layer, block, tier)
        return k.to(device, non_blocking=True), v.to(device, non_blocking=True)

    def close(self) -> None:
        """Close the NVMe tier's files (the data stays on disk)."""
        buf = self._buffers.get(MemoryTier.NVME)
        if isinstance(buf, _FileTier):
            buf.close()
            del self._buffers[MemoryTier.NVME]

    def __repr__(self) -> str:  # pragma: no cover
        return f"TieredStorage(tiers=[{','.join(t.value for t in self.tiers)}], blocks={self.max_blocks})"


class TierMover:
    """Runs a storage's batched block moves, on a side CUDA stream of its
    own when ``asynchronous`` (and CUDA is up) so the caller's stream never
    waits for them: the side stream first waits for the work already queued
    on the caller's stream (which may still read the source blocks), then
    copies; :meth:`fence` makes the caller's stream wait for every move
    issued so far.  The tier directory is updated when a move is issued."""

    def __init__(self, storage, *, asynchronous: bool) -> None:
        self.storage = storage
        self.asynchronous = asynchronous
        self._side = None

    def _stream(self):
        import torch
        if not (self.asynchronous and torch.cuda.is_available()):
            return None
        if self._side is None:
            self._side = torch.cuda.Stream()
        return self._side

    def move(self, layer: int, blocks, src, dst) -> int:
        import torch
        side = self._stream()
        if side is None:
            return self.storage.move_blocks(layer=layer, blocks=blocks, src=src, dst=dst)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            return self.storage.move_blocks(layer=layer, blocks=blocks, src=src, dst=dst)

    def fence(self) -> None:
        import torch
        if self._side is not None:
            torch.cuda.current_stream().wait_stream(self._side)


__all__ = ["MemoryTier", "TieredStorage", "TierMover"]
