"""Host logic of the sequence-sharded decode on CPU with world_size-2 gloo
ranks: the chunk partition, the all-gather of fp32 (o, lse) partials
(halo_b200.sharded.gather_partials) and the LSE merge of the gathered parts
in rank order reproduce single-process attention over the whole context.
The per-rank partials come from the CPU oracle (no GPU here)."""
from __future__ import annotations

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from halo_b200.sharded import shard_range

WORLD = 2


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs():
    g = torch.Generator().manual_seed(123)
    B, H, H_kv, D, T, C = 2, 8, 2, 64, 1000, 96
    q = torch.randn(B, H, 1, D, generator=g)
    k = torch.randn(B, H_kv, T, D, generator=g)
    v = torch.randn(B, H_kv, T, D, generator=g)
    return q, k, v, C


def _rank_main(rank: int, port: int, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        from oracle import attention as OA
        from halo_b200.sharded import gather_partials
        q, k, v, C = _inputs()
        n_chunks = -(-k.shape[-2] // C)
        lo, hi = shard_range(n_chunks, WORLD, rank)
        chunks = [(k[..., a * C:min((a + 1) * C, k.shape[-2]), :],
                   v[..., a * C:min((a + 1) * C, k.shape[-2]), :], a * C, False)
                  for a in range(lo, hi)]
        out, lse = OA.chunked_attention(q, chunks)
        lse_parts, o_parts = gather_partials(out[:, :, 0].contiguous().float(),
                                             lse[:, :, 0].contiguous().float())
        # fold the parts in rank order with the oracle's pairwise merge
        o, l = o_parts[0].unsqueeze(2), lse_parts[0].unsqueeze(2)
        for r in range(1, WORLD):
            o, l = OA.lse_merge(o, l, o_parts[r].unsqueeze(2), lse_parts[r].unsqueeze(2))
        result_q.put((rank, o.clone(), l.clone(), (lo, hi)))
    finally:
        dist.destroy_process_group()


def test_shard_range_partitions_every_chunk_once():
    for n in (1, 7, 64, 256, 1000):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (a, b), (c, d) in zip(ranges, ranges[1:]):
                assert b == c
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_two_gloo_ranks_gather_and_merge_equal_full_attention():
    from oracle import attention as OA
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, result_q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [result_q.get(timeout=120) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v, _ = _inputs()
    ro, rl = OA.full_attention_f64(q, k, v)
    shards = sorted(r[3] for r in results)
    assert shards[0][0] == 0 and shards[0][1] == shards[1][0]
    for rank, o, l, _ in results:
        # every rank holds the same merged result
        assert (o.double() - ro).abs().max().item() <= 1e-5
        assert (l.double() - rl).abs().max().item() <= 1e-5


def test_sharded_kivi_decoder_rejects_bad_arguments():
    """The sharded KIVI decoder checks its exchange and that each shard is a
    whole number of quantisation groups before touching a device."""
    import pytest
    import torch
    from halo_b200.sharded import ShardedKiviDecoder
    k = torch.zeros(1, 2, 64, 128, dtype=torch.float16)
    with pytest.raises(ValueError, match="exchange"):
        ShardedKiviDecoder(k, k, exchange="mpi")
    with pytest.raises(ValueError, match="group_size"):
        ShardedKiviDecoder(k[..., :48, :], k[..., :48, :], group_size=32)
