"""Sequence-sharded decode on 2 GPUs (NCCL): each rank decodes its shard of
the chunks, the fp32 (o, lse) partials are all-gathered and LSE-merged; the
result equals single-GPU decode over the whole context and the oracle.
Skipped on boxes with fewer than 2 GPUs."""
from __future__ import annotations

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(large=False):
    g = torch.Generator().manual_seed(321 + large)
    # large: a cfg5-shaped shard per rank, long enough for the single-launch
    # fused decode + exchange (dynamic schedule); small: split-KV + kx_kernel
    B, H, H_kv, D, T, C = (1, 64, 8, 128, 65536, 4096) if large else (2, 16, 4, 128, 24576, 4096)
    q = torch.randn(B, H, D, generator=g).bfloat16()
    k = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    v = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    return q, k, v, C


def _rank_main(rank: int, port: int, result_q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from halo_b200.sharded import ShardedDecoder, shard_range
        dev = torch.device("cuda", rank)
        res = {}
        for large in (False, True):
            q, k, v, C = _inputs(large)
            lo, hi = shard_range(k.shape[-2] // C, WORLD, rank)
            ks = k[..., lo * C:hi * C, :].to(dev)
            vs = v[..., lo * C:hi * C, :].to(dev)
            for mode in ("p2p", "nccl"):
                dec = ShardedDecoder(ks, vs, start=lo * C, chunk_size=C, group=dist.group.WORLD,
                                     exchange=mode)
                lse = torch.empty(q.shape[:2], device=dev)
                for _ in range(3):   # repeated calls cycle the exchange epochs
                    out, _ = dec(q.to(dev), out=torch.empty(q.shape, device=dev), lse=lse)
                torch.cuda.synchronize()
                res[(large, mode)] = (out.cpu(), lse.cpu())
                if mode == "p2p":   # a captured step replays in step across ranks
                    o_g = torch.empty(q.shape, device=dev)
                    l_g = torch.empty(q.shape[:2], device=dev)
                    graph = dec.capture(q.to(dev), out=o_g, lse=l_g)
                    for _ in range(3):
                        graph.replay()
                    torch.cuda.synchronize()
                    res[(large, "graph")] = (o_g.cpu(), l_g.cpu())
                    del graph
                dec.close()
        from halo_b200 import _lib as L
        result_q.put((rank, res, L.device_error()))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_sharded_decode_two_gpus_matches_single_gpu_and_oracle():
    import torch.multiprocessing as mp
    from halo_b200 import ops
    from oracle import attention as OA
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, result_q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [result_q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for large in (False, True):
        q, k, v, C = _inputs(large)
        G = q.shape[1] // k.shape[1]
        chunks = [(k[..., a:a + C, :].cuda(), v[..., a:a + C, :].cuda(), a, False)
                  for a in range(0, k.shape[-2], C)]
        o1, l1 = ops.chunked_decode(q.cuda(), chunks, out_dtype=torch.float32)
        for hk in range(k.shape[1]):   # oracle one kv-head group at a time
            hs = slice(hk * G, (hk + 1) * G)
            ro, rl = OA.full_attention_f64(q[:, hs].unsqueeze(2), k[:, hk:hk + 1], v[:, hk:hk + 1])
            for rank, res, err in results:
                assert err == 0
                for key, (out, lse) in res.items():
                    if key[0] != large:
                        continue
                    assert (out[:, hs].double() - ro[:, :, 0]).abs().max().item() <= 2e-3, key
                    assert (lse[:, hs].double() - rl[:, :, 0]).abs().max().item() <= 1e-4, key
        for rank, res, err in results:
            for key, (out, lse) in res.items():
                if key[0] == large:
                    assert (out - o1.cpu()).abs().max().item() <= 1e-5, key
