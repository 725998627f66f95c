"""The NVMe tier of TieredStorage (``halo/memory_tier.py:61-103, 228-258``):
raw-byte block files, any dtype bit-exact, the files sized for every slot,
blocks moved down the tier ladder and back (the scenarios of the reference's
tests/test_memmap_nvme.py), plus the positioned-read refetch path."""
from __future__ import annotations

import os

import pytest
import torch

from halo_b200.memory_tier import MemoryTier, TieredStorage


def _storage(tmp_path, tiers, dtype=torch.float32, L=2, H_kv=2, D=8, block=4, blocks=4):
    return TieredStorage(tiers=tiers, num_layers=L, num_kv_heads=H_kv, head_dim=D,
                         block_size=block, dtype=dtype, device=torch.device("cpu"),
                         max_blocks=blocks, nvme_path=str(tmp_path / "nvme"))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_nvme_blocks_round_trip_bit_exact(tmp_path, dtype):
    st = _storage(tmp_path, [MemoryTier.GPU, MemoryTier.NVME], dtype=dtype)
    g = torch.Generator().manual_seed(1)
    blocks = {}
    for layer, b in ((1, 2), (0, 0), (1, 3)):
        k = torch.randn(2, 4, 8, generator=g).to(dtype)
        v = torch.randn(2, 4, 8, generator=g).to(dtype)
        st.write_new_block(layer=layer, block=b, keys=k, values=v, tier="nvme")
        blocks[(layer, b)] = (k, v)
    for (layer, b), (k, v) in blocks.items():
        assert st.locate_block(layer=layer, block=b) == "nvme"
        rk, rv = st.read_block(layer=layer, block=b)
        assert rk.dtype == dtype and rk.shape == (2, 4, 8)
        assert torch.equal(rk.view(torch.uint8), k.view(torch.uint8))
        assert torch.equal(rv.view(torch.uint8), v.view(torch.uint8))
    st.close()


def test_nvme_files_sized_for_every_slot(tmp_path):
    st = _storage(tmp_path, [MemoryTier.GPU, MemoryTier.NVME], L=1, H_kv=2, D=4, block=2,
                  blocks=2)
    k = torch.arange(16, dtype=torch.float32).reshape(2, 2, 4)
    st.write_new_block(layer=0, block=0, keys=k, values=k.clone(), tier="nvme")
    expected = 1 * 2 * 2 * 2 * 4 * 4   # layers x blocks x heads x rows x dim x bytes
    assert os.path.getsize(tmp_path / "nvme" / "keys.bin") == expected
    assert os.path.getsize(tmp_path / "nvme" / "values.bin") == expected
    st.close()


def test_block_moves_down_the_ladder_and_back(tmp_path):
    st = _storage(tmp_path, ["gpu", "dram", "nvme"], L=1, H_kv=1, D=4, block=2, blocks=2)
    k = torch.tensor([[[1.0, 2.0, 3.0, 4.0], [5.0, 6.0, 7.0, 8.0]]])
    st.write_new_block(layer=0, block=1, keys=k, values=-k, tier="gpu")
    st.move_block(layer=0, block=1, src="gpu", dst="dram")
    st.move_block(layer=0, block=1, src="dram", dst="nvme")
    assert st.locate_block(layer=0, block=1) == "nvme"
    rk, rv = st.read_block(layer=0, block=1)
    assert torch.equal(rk, k) and torch.equal(rv, -k)
    rk, rv = st.refetch_block(layer=0, block=1, device=torch.device("cpu"))
    assert torch.equal(rk, k) and torch.equal(rv, -k)
    st.move_block(layer=0, block=1, src="nvme", dst="gpu")
    assert st.locate_block(layer=0, block=1) == "gpu"
    rk, _ = st.read_block(layer=0, block=1)
    assert torch.equal(rk, k)
    st.close()


def test_nvme_tier_refuses_blocks_outside_its_slots(tmp_path):
    st = _storage(tmp_path, ["gpu", "nvme"], blocks=2)
    with pytest.raises(IndexError):
        st.write_new_block(layer=0, block=2, keys=torch.zeros(2, 4, 8), values=torch.zeros(2, 4, 8),
                           tier="nvme")
    st.close()


def test_unrequested_tier_is_refused(tmp_path):
    st = _storage(tmp_path, ["gpu", "dram"])
    with pytest.raises(ValueError):
        st.write_new_block(layer=0, block=0, keys=torch.zeros(2, 4, 8),
                           values=torch.zeros(2, 4, 8), tier="nvme")
