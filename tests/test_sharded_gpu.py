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


def _kivi_inputs():
    """A cfg4-shaped KIVI cache cut short: B2, 32 q-heads / 8 KV heads,
    D 128, 8192 quantised rows + 128 fp16 recent rows, keys with outlier
    channels."""
    g = torch.Generator().manual_seed(555)
    B, H, H_kv, D, T, R = 2, 32, 8, 128, 8192, 128
    q = torch.randn(B, H, D, generator=g).half()
    k = torch.randn(B, H_kv, T + R, D, generator=g)
    for h in range(H_kv):
        k[:, h, :, torch.randperm(D, generator=g)[:4]] *= 10
    v = torch.randn(B, H_kv, T + R, D, generator=g).half()
    return q, k.half(), v, T


def _kivi_rank_main(rank: int, port: int, result_q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from halo_b200.sharded import ShardedKiviDecoder
        dev = torch.device("cuda", rank)
        q, k, v, T = _kivi_inputs()
        lo, hi = rank * T // WORLD, (rank + 1) * T // WORLD
        last = rank == WORLD - 1
        outs = []
        for mode in ("p2p", "nccl"):
            dec = ShardedKiviDecoder(k[..., lo:hi, :].to(dev), v[..., lo:hi, :].to(dev), bits=2,
                                     group_size=32,
                                     recent_k=k[..., T:, :].to(dev) if last else None,
                                     recent_v=v[..., T:, :].to(dev) if last else None,
                                     exchange=mode)
            for _ in range(2):   # repeated calls cycle the exchange epochs
                out, lse = dec(q.to(dev))
                torch.cuda.synchronize()
                outs.append((out.float().cpu(), lse.cpu()))
            dec.close()
        from halo_b200 import _lib as L
        result_q.put((rank, outs, L.device_error()))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_sharded_kivi_decode_two_gpus_matches_single_gpu():
    """Two ranks, each with half of the quantised rows (the second also the
    16-bit recent rows), with the NVLink and the NCCL exchange, against one
    KIVICache over the whole context on one GPU (same codes, since
    quantisation is per row) and a float64 attention over the dequantised
    keys and values."""
    import math
    import torch.multiprocessing as mp
    from halo_b200.baselines.kivi_cache import KIVICache, dequantize_packed
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_kivi_rank_main, args=(r, port, result_q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [result_q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    q, k, v, T = _kivi_inputs()
    cache = KIVICache(bits=2, group_size=32, residual_length=128, fused_attention=True)
    cache.update(k.cuda(), v.cuda(), layer_idx=0)
    ref = cache.compute_attention(q.cuda().unsqueeze(2), layer_idx=0).squeeze(2).float().cpu()
    kq, vq = cache._k_quant[0], cache._v_quant[0]
    kd = dequantize_packed(kq.codes[:, :, :kq.T], kq.scale[:, :, :kq.T], kq.zero[:, :, :kq.T],
                           bits=2, group_size=32)
    vd = dequantize_packed(vq.codes[:, :, :vq.T], vq.scale[:, :, :vq.T], vq.zero[:, :, :vq.T],
                           bits=2, group_size=32)
    G = q.shape[1] // k.shape[1]
    kf = torch.cat([kd, cache._k_recent[0]], 2).double().cpu().repeat_interleave(G, 1)
    vf = torch.cat([vd, cache._v_recent[0]], 2).double().cpu().repeat_interleave(G, 1)
    s = (q.double().unsqueeze(2) @ kf.transpose(-1, -2)).squeeze(2) / math.sqrt(q.shape[-1])
    f64 = (torch.softmax(s, -1).unsqueeze(2) @ vf).squeeze(2)
    lse64 = torch.logsumexp(s, -1)
    for rank, outs, err in results:
        assert err == 0
        for out, lse in outs:
            assert (out - ref).abs().max().item() <= 2e-3
            assert (out.double() - f64).abs().max().item() <= 2e-3
            assert (lse.double() - lse64).abs().max().item() <= 1e-4
