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


def _inputs():
    g = torch.Generator().manual_seed(321)
    B, H, H_kv, D, T, C = 2, 16, 4, 128, 24576, 4096
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
        q, k, v, C = _inputs()
        lo, hi = shard_range(k.shape[-2] // C, WORLD, rank)
        dev = torch.device("cuda", rank)
        ks = k[..., lo * C:hi * C, :].to(dev)
        vs = v[..., lo * C:hi * C, :].to(dev)
        res = {}
        for mode in ("p2p", "nccl"):
            dec = ShardedDecoder(ks, vs, start=lo * C, chunk_size=C, group=dist.group.WORLD,
                                 exchange=mode)
            lse = torch.empty(q.shape[:2], device=dev)
            for _ in range(3):   # repeated calls cycle the exchange epochs
                out, _ = dec(q.to(dev), out=torch.empty(q.shape, device=dev), lse=lse)
            torch.cuda.synchronize()
            res[mode] = (out.cpu(), lse.cpu())
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
    q, k, v, C = _inputs()
    ro, rl = OA.full_attention_f64(q.unsqueeze(2), k, v)
    chunks = [(k[..., a:a + C, :].cuda(), v[..., a:a + C, :].cuda(), a, False)
              for a in range(0, k.shape[-2], C)]
    o1, l1 = ops.chunked_decode(q.cuda(), chunks, out_dtype=torch.float32)
    for rank, res, err in results:
        assert err == 0
        for mode, (out, lse) in res.items():
            assert (out.double() - ro[:, :, 0]).abs().max().item() <= 2e-3, mode
            assert (lse.double() - rl[:, :, 0]).abs().max().item() <= 1e-4, mode
            assert (out - o1.cpu()).abs().max().item() <= 1e-5, mode
