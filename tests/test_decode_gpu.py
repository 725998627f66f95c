"""GPU parity: split-KV decode + LSE merge (sm_100a) vs the CPU oracle and the
reference's golden vectors.

Tolerances: attention output within 2e-3 max-abs of the
fp32 reference for 16-bit inputs (compared on the fp32 output, before any
rounding to the storage dtype), LSE within 1e-4; fp32 inputs within 1e-5.
"""
from __future__ import annotations

import math
import random

import pytest
import torch

import inputs as I
from oracle import attention as OA

pytestmark = pytest.mark.gpu

OUT_TOL_16 = 2e-3
LSE_TOL = 1e-4
OUT_TOL_32 = 1e-5


def _tol(dtype):
    return OUT_TOL_32 if dtype == torch.float32 else OUT_TOL_16


def _ops():
    from halo_b200 import ops
    return ops


def _gpu_chunks(k, v, bounds, causal=False, dev="cuda"):
    kd, vd = k.to(dev), v.to(dev)
    return [(kd[..., a:b, :], vd[..., a:b, :], a, causal) for a, b in bounds]


def _bounds(T, chunk):
    return [(c0, min(c0 + chunk, T)) for c0 in range(0, T, chunk)]


@pytest.mark.parametrize("name", list(I.WALK_CASES))
def test_decode_matches_reference_golden(cuda_device, name):
    ops = _ops()
    (q, k, v), chunk = I.walk_inputs(name)
    g = I.load("attention.npz")[name]
    chunks = _gpu_chunks(k, v, _bounds(k.shape[-2], chunk))
    out, lse = ops.chunked_decode(q.to(cuda_device), chunks, out_dtype=torch.float32)
    ref_o = torch.from_numpy(g["out"])[:, :, 0]
    ref_l = torch.from_numpy(g["lse"])[:, :, 0]
    assert (out.cpu() - ref_o).abs().max().item() <= _tol(q.dtype)
    assert (lse.cpu() - ref_l).abs().max().item() <= LSE_TOL
    # output in q.dtype equals the fp32 result rounded once
    out_q, _ = ops.chunked_decode(q.to(cuda_device), chunks)
    assert out_q.dtype == q.dtype
    torch.testing.assert_close(out_q.float(), out.to(q.dtype).float(), rtol=0, atol=0)


def test_decode_config1_full(cuda_device):
    """The fp32 CPU-runnable decode case at full size (B1, H32/8, D128, T8192,
    16 chunks of 512, hot chunks {0, 13, 14, 15} walked first)."""
    ops = _ops()
    g = I.load("config1.npz")["config1"]
    q, k, v = I.config1_inputs()
    order = [int(c) for c in g["order"]]
    chunks = _gpu_chunks(k, v, [(c * 512, (c + 1) * 512) for c in order])
    out, lse = ops.chunked_decode(q.to(cuda_device), chunks)
    assert (out.cpu() - torch.from_numpy(g["out"])).abs().max().item() <= OUT_TOL_32 * 10
    assert (lse.cpu() - torch.from_numpy(g["lse"])).abs().max().item() <= LSE_TOL


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("chunk_size", [128, 512])
def test_decode_small_gqa(cuda_device, dtype, chunk_size):
    """Mirrors the reference Triton test (1K cache, GQA 4:1, D 64) with the
    reference's relative-L2 bounds, plus the absolute/LSE bounds."""
    ops = _ops()
    torch.manual_seed(0)
    B, H, H_kv, D, T = 1, 8, 2, 64, 1024
    q = (torch.randn(B, H, 1, D) * 0.1).to(dtype)
    k = (torch.randn(B, H_kv, T, D) * 0.1).to(dtype)
    v = (torch.randn(B, H_kv, T, D) * 0.1).to(dtype)
    ref_o, ref_l = OA.full_attention_f64(q, k, v, q_pos=T - 1)
    chunks = _gpu_chunks(k, v, _bounds(T, chunk_size), causal=True)
    qp = torch.tensor([T - 1], device=cuda_device)
    out, lse = ops.chunked_decode(q.to(cuda_device), chunks, q_pos=qp, out_dtype=torch.float32)
    rel = ((out.cpu().double() - ref_o[:, :, 0]).norm() / ref_o.norm()).item()
    assert rel <= (1e-4 if dtype == torch.float32 else 5e-3)
    assert (out.cpu().double() - ref_o[:, :, 0]).abs().max().item() <= _tol(dtype)
    assert (lse.cpu().double() - ref_l[:, :, 0]).abs().max().item() <= LSE_TOL


@pytest.mark.parametrize("chunk_size", [256, 512])
def test_decode_causal_mask_and_truncation(cuda_device, chunk_size):
    ops = _ops()
    torch.manual_seed(1)
    B, H, H_kv, D, T = 1, 4, 1, 64, 2048
    q = torch.randn(B, H, 1, D) * 0.1
    k = torch.randn(B, H_kv, T, D) * 0.1
    v = torch.randn(B, H_kv, T, D) * 0.1
    qp = torch.tensor([T // 2], device=cuda_device)
    ref_o, _ = OA.full_attention_f64(q, k, v, q_pos=T // 2)
    out, _ = ops.chunked_decode(q.to(cuda_device), _gpu_chunks(k, v, _bounds(T, chunk_size), True),
                                q_pos=qp)
    assert ((out.cpu().double() - ref_o[:, :, 0]).norm() / ref_o.norm()).item() <= 1e-4
    half, _ = ops.chunked_decode(q.to(cuda_device), _gpu_chunks(k, v, [(0, T // 2 + 1)], True),
                                 q_pos=qp)
    assert ((out - half).norm() / out.norm()).item() <= 1e-5


def test_decode_noncontiguous_partition_and_permutation(cuda_device):
    ops = _ops()
    torch.manual_seed(4)
    B, H, H_kv, D, T = 1, 8, 2, 64, 2048
    q = torch.randn(B, H, 1, D) * 0.1
    k = torch.randn(B, H_kv, T, D) * 0.1
    v = torch.randn(B, H_kv, T, D) * 0.1
    intervals = [(0, 256), (768, 1024), (1280, 1408), (1536, 1664), (1856, 2048)]
    keep = torch.zeros(T, dtype=torch.bool)
    for a, b in intervals:
        keep[a:b] = True
    ref_o, ref_l = OA.full_attention_f64(q, k, v, q_pos=T - 1, keep=keep)
    qp = torch.tensor([T - 1], device=cuda_device)
    chunks = _gpu_chunks(k, v, intervals, True)
    out, lse = ops.chunked_decode(q.to(cuda_device), chunks, q_pos=qp)
    assert ((out.cpu().double() - ref_o[:, :, 0]).norm() / ref_o.norm()).item() <= 1e-4
    random.seed(0)
    perm = chunks.copy()
    random.shuffle(perm)
    out_p, lse_p = ops.chunked_decode(q.to(cuda_device), perm, q_pos=qp)
    assert ((out_p.cpu().double() - ref_o[:, :, 0]).norm() / ref_o.norm()).item() <= 1e-4
    assert (lse_p - lse).abs().max().item() <= 1e-5


def test_decode_per_batch_q_pos_and_fully_masked_rows(cuda_device):
    """Per-row causal positions, including a row that sees no key at all
    (output zeros, lse -inf, like finalize's safe divide)."""
    ops = _ops()
    torch.manual_seed(5)
    B, H, H_kv, D, T = 3, 8, 2, 128, 700
    q = torch.randn(B, H, 1, D).bfloat16()
    k = torch.randn(B, H_kv, T, D).bfloat16()
    v = torch.randn(B, H_kv, T, D).bfloat16()
    qpos = [T - 1, 333, -1]
    chunks = _gpu_chunks(k, v, [(100, T)], True)   # keys start at 100 -> row 2 sees nothing
    out, lse = ops.chunked_decode(q.to(cuda_device), chunks,
                                  q_pos=torch.tensor(qpos, device=cuda_device),
                                  out_dtype=torch.float32)
    for b in range(2):
        keep = torch.zeros(T, dtype=torch.bool)
        keep[100:] = True
        ro, rl = OA.full_attention_f64(q[b:b + 1], k[b:b + 1], v[b:b + 1], q_pos=qpos[b], keep=keep)
        assert (out[b].cpu().double() - ro[0, :, 0]).abs().max().item() <= OUT_TOL_16
        assert (lse[b].cpu().double() - rl[0, :, 0]).abs().max().item() <= LSE_TOL
    assert torch.all(out[2] == 0)
    assert torch.all(torch.isneginf(lse[2]))


def test_decode_empty_inputs(cuda_device):
    ops = _ops()
    q = torch.randn(2, 4, 1, 64, device=cuda_device, dtype=torch.bfloat16)
    out, lse = ops.chunked_decode(q, [])
    assert torch.all(out == 0) and torch.all(torch.isneginf(lse))
    k = torch.empty(2, 2, 0, 64, device=cuda_device, dtype=torch.bfloat16)
    out, lse = ops.chunked_decode(q, [(k, k, 0, True)])
    assert torch.all(out == 0) and torch.all(torch.isneginf(lse))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_accumulate_matches_triton_state(cuda_device, dtype):
    """ACCUMULATE mode keeps the (m, l, o) state of halo/triton_chunked.py."""
    ops = _ops()
    (q, k, v), chunk = I.walk_inputs("walk_f32_gqa4")
    q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
    bounds = _bounds(k.shape[-2], chunk)
    qp = torch.full((q.shape[0],), 150, device=cuda_device)
    B, H, D = q.shape[0], q.shape[1], q.shape[-1]
    m = torch.full((B, H), float("-inf"), device=cuda_device)
    l = torch.zeros(B, H, device=cuda_device)
    o = torch.zeros(B, H, D, device=cuda_device)
    for a, b in bounds:
        ops.accumulate_decode(q.to(cuda_device), _gpu_chunks(k, v, [(a, b)], True), m, l, o,
                              scale=1 / math.sqrt(D), q_pos=qp)
    rm, rl, ro = OA.acc_state_from_chunks(q, [(k[..., a:b, :], v[..., a:b, :], a, True)
                                              for a, b in bounds], q_pos=150)
    assert (m.cpu() - rm[..., 0]).abs().max().item() <= 1e-5
    finite = torch.isfinite(rm[..., 0])
    torch.testing.assert_close((o / l.unsqueeze(-1)).cpu()[finite],
                               (ro / rl.unsqueeze(-1))[..., 0, :][finite],
                               atol=_tol(dtype), rtol=0)


@pytest.mark.parametrize("name", list(I.PREFILL_CASES))
def test_multi_query_causal_matches_reference(cuda_device, name):
    ops = _ops()
    (q, k, v), T_cold, chunk = I.prefill_inputs(name)
    g = I.load("attention.npz")[name]
    T, T_q = k.shape[-2], q.shape[-2]
    chunks = _gpu_chunks(k, v, _bounds(T, chunk), True)
    out, lse = ops.multi_query_attention(q.to(cuda_device), chunks, query_pos_offset=T - T_q,
                                         out_dtype=torch.float32)
    assert (out.cpu() - torch.from_numpy(g["out"])).abs().max().item() <= _tol(q.dtype)
    assert (lse.cpu() - torch.from_numpy(g["lse"])).abs().max().item() <= LSE_TOL


def test_lse_merge_parts(cuda_device):
    ops = _ops()
    torch.manual_seed(9)
    B, H, D, T = 2, 8, 128, 1500
    q = torch.randn(B, H, 1, D)
    k = torch.randn(B, 2, T, D)
    v = torch.randn(B, 2, T, D)
    parts = [(0, 400), (400, 401), (401, 1500)]
    ms, ls, os_ = [], [], []
    for a, b in parts:
        m, l, o = OA.acc_state_from_chunks(q, [(k[..., a:b, :], v[..., a:b, :], a, False)])
        ms.append(m[..., 0]); ls.append(l[..., 0]); os_.append(o[..., 0, :])
    # a fully masked part contributes nothing
    ms.append(torch.full((B, H), float("-inf"))); ls.append(torch.zeros(B, H)); os_.append(torch.zeros(B, H, D))
    mp = torch.stack(ms, -1).contiguous().to(cuda_device)
    lp = torch.stack(ls, -1).contiguous().to(cuda_device)
    op = torch.stack(os_, -2).contiguous().to(cuda_device)
    out, lse = ops.lse_merge(mp, lp, op)
    ro, rl = OA.full_attention_f64(q, k, v)
    assert (out.cpu().double() - ro[:, :, 0]).abs().max().item() <= 1e-5
    assert (lse.cpu().double() - rl[:, :, 0]).abs().max().item() <= 1e-5


def _random_parts(B, H, P, Dv, seed):
    """Synthetic partial states (natural-log max m, weight l, unnormalised
    output o), a few parts fully masked (m = -inf, l = 0, o = 0)."""
    g = torch.Generator().manual_seed(seed)
    m = torch.randn(B, H, P, generator=g) * 3
    l = torch.rand(B, H, P, generator=g) * 50 + 0.5
    o = torch.randn(B, H, P, Dv, generator=g) * l.unsqueeze(-1)
    dead = torch.rand(B, H, P, generator=g) < 0.2
    dead[..., 0] = False                      # every row keeps one live part
    m[dead], l[dead] = float("-inf"), 0.0
    o[dead] = 0.0
    return m, l, o


def _merge_f64(m, l, o):
    md, ld, od = m.double(), l.double(), o.double()
    M = md.amax(-1, keepdim=True)
    w = torch.where(torch.isneginf(md), torch.zeros_like(md), torch.exp(md - M))
    L = (w * ld).sum(-1)
    return (w.unsqueeze(-1) * od).sum(-2) / L.unsqueeze(-1), M.squeeze(-1) + torch.log(L)


@pytest.mark.parametrize("Dv", [192, 256])
@pytest.mark.parametrize("P", [3, 37])
def test_lse_merge_wide_rows(cuda_device, Dv, P):
    """Rows wider than 128 columns (eight a lane, partials folded 16 per
    memory round trip): the P-way merge equals a float64 merge."""
    ops = _ops()
    B, H = 2, 8
    m, l, o = _random_parts(B, H, P, Dv, seed=Dv + P)
    out, lse = ops.lse_merge(m.to(cuda_device), l.to(cuda_device), o.to(cuda_device))
    ro, rl = _merge_f64(m, l, o)
    assert (out.cpu().double() - ro).abs().max().item() <= 1e-5
    assert (lse.cpu().double() - rl).abs().max().item() <= 1e-5


@pytest.mark.parametrize("Dv", [128, 256])
def test_sharded_merge_single_rank(cuda_device, Dv):
    """halo_sharded_merge with a world of one (no peer traffic): the local
    merge, the exchange through this rank's own buffer and the fold give
    the plain merge; two calls cover both epoch parities of the buffer."""
    import ctypes
    from halo_b200 import _lib as L
    lib = L.lib()
    B, H, P = 1, 8, 21
    m, l, o = _random_parts(B, H, P, Dv, seed=3 * Dv)
    md, ld, od = (t.contiguous().to(cuda_device) for t in (m, l, o))
    nbytes = lib.halo_exchange_bytes(1, B * H, Dv)
    assert nbytes > 0
    buf = torch.zeros(nbytes, dtype=torch.uint8, device=cuda_device)
    bufs = (ctypes.c_void_p * 1)(buf.data_ptr())
    ro, rl = _merge_f64(m, l, o)
    for _ in range(2):
        out = torch.full((B, H, Dv), float("nan"), device=cuda_device)
        lse = torch.full((B, H), float("nan"), device=cuda_device)
        rc = lib.halo_sharded_merge(B, H, Dv, P, md.data_ptr(), ld.data_ptr(), od.data_ptr(), 1, P,
                                    Dv, P * Dv, 1, 0, bufs, L.DTYPE_F32, out.data_ptr(),
                                    out.stride(0), out.stride(1), lse.data_ptr(),
                                    L.stream_handle(cuda_device))
        L.check(rc, "halo_sharded_merge")
        torch.cuda.synchronize()
        assert L.device_error() == 0
        assert (out.cpu().double() - ro).abs().max().item() <= 1e-5
        assert (lse.cpu().double() - rl).abs().max().item() <= 1e-5


def test_large_context_properties(cuda_device):
    """Config-5-like context at reduced heads: chunk-order invariance and
    linearity in V (attention is linear in V for fixed q, k)."""
    ops = _ops()
    torch.manual_seed(12)
    B, H, H_kv, D, T, chunk = 1, 16, 2, 128, 131072, 4096
    dev = cuda_device
    q = torch.randn(B, H, 1, D, device=dev).bfloat16()
    k = torch.randn(B, H_kv, T, D, device=dev).bfloat16()
    v = torch.randn(B, H_kv, T, D, device=dev).bfloat16()
    ch = [(k[..., a:b, :], v[..., a:b, :], a, False) for a, b in _bounds(T, chunk)]
    o1, l1 = ops.chunked_decode(q, ch, out_dtype=torch.float32)
    o2, l2 = ops.chunked_decode(q, ch[::-1], out_dtype=torch.float32)
    assert (o1 - o2).abs().max().item() <= 1e-5 and (l1 - l2).abs().max().item() <= 1e-5
    v2 = (v.float() * 2).bfloat16()     # exact doubling
    ch2 = [(k[..., a:b, :], v2[..., a:b, :], a, False) for a, b in _bounds(T, chunk)]
    o3, l3 = ops.chunked_decode(q, ch2, out_dtype=torch.float32)
    # the default (dynamic) schedule may fold the keys in a different order
    # from call to call: equal up to fp32 rounding
    assert (o3 - 2 * o1).abs().max().item() <= 1e-5 and (l3 - l1).abs().max().item() <= 1e-6
    # the static split (max_split_rows > 0) is deterministic: bit-identical
    s1 = ops.chunked_decode(q, ch, out_dtype=torch.float32, max_split_rows=4096)
    s3 = ops.chunked_decode(q, ch2, out_dtype=torch.float32, max_split_rows=4096)
    assert torch.equal(s3[1], s1[1]) and torch.equal(s3[0], 2 * s1[0])
    assert (s1[0] - o1).abs().max().item() <= 1e-5
    # spot-check one kv-head group against the fp64 oracle
    ro, rl = OA.full_attention_f64(q[:, :8].cpu(), k[:, :1].cpu(), v[:, :1].cpu())
    assert (o1[:, :8].cpu().double() - ro[:, :, 0]).abs().max().item() <= OUT_TOL_16
    assert (l1[:, :8].cpu().double() - rl[:, :, 0]).abs().max().item() <= LSE_TOL


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("layout", ["contiguous", "causal", "scattered"])
def test_decode_dynamic_schedule(cuda_device, dtype, layout):
    """Contexts long enough for the dynamic schedule (pieces taken at run
    time by groups of CTAs per kv-head): parity with the oracle and with the
    static split, per-batch causal positions, chunks from separate buffers
    (one segment each), repeated calls (the counters are reset by the
    kernel), and the workspace control block left zero."""
    ops = _ops()
    from halo_b200 import _lib as L
    g = torch.Generator().manual_seed(77)
    B, H, H_kv, D, T, chunk = 2, 64, 8, 128, 32768, 4096
    q = torch.randn(B, H, 1, D, generator=g).to(dtype)
    k = torch.randn(B, H_kv, T, D, generator=g)
    k[..., torch.randperm(D, generator=g)[:4]] *= 10
    k, v = k.to(dtype), torch.randn(B, H_kv, T, D, generator=g).to(dtype)
    dev = cuda_device
    causal = layout != "contiguous"
    if layout == "scattered":   # every chunk its own allocation
        ch = [(k[..., a:b, :].to(dev).contiguous(), v[..., a:b, :].to(dev).contiguous(), a, True)
              for a, b in _bounds(T, chunk)]
    else:
        ch = _gpu_chunks(k, v, _bounds(T, chunk), causal=causal, dev=dev)
    q_pos = torch.tensor([T - 1, 20000], device=dev) if causal else None
    qd = q.to(dev)
    outs = [ops.chunked_decode(qd, ch, q_pos=q_pos, out_dtype=torch.float32) for _ in range(3)]
    st = ops.chunked_decode(qd, ch, q_pos=q_pos, out_dtype=torch.float32, max_split_rows=2048)
    G = H // H_kv
    for b in range(B):
        qp = (T - 1 if b == 0 else 20000) if causal else None
        for hk in range(H_kv):      # one kv-head group at a time (oracle memory)
            hs = slice(hk * G, (hk + 1) * G)
            ro, rl = OA.full_attention_f64(q[b:b + 1, hs], k[b:b + 1, hk:hk + 1],
                                           v[b:b + 1, hk:hk + 1], q_pos=qp)
            for out, lse in outs + [st]:
                assert (out[b:b + 1, hs].cpu().double() - ro[:, :, 0]).abs().max().item() \
                    <= OUT_TOL_16
                assert (lse[b:b + 1, hs].cpu().double() - rl[:, :, 0]).abs().max().item() \
                    <= LSE_TOL
    for out, lse in outs:
        assert (out - st[0]).abs().max().item() <= 1e-5
    # ACCUMULATE over two halves (each long enough for the in-kernel merge)
    # then a FINALIZE with that prior state equals the one-call result
    m = torch.full((B, H), float("-inf"), device=dev)
    l = torch.zeros(B, H, device=dev)
    o = torch.zeros(B, H, D, device=dev)
    half = len(ch) // 2
    ops.accumulate_decode(qd, ch[:half], m, l, o, scale=1 / math.sqrt(D), q_pos=q_pos)
    o2, l2 = ops.chunked_decode(qd, ch[half:], q_pos=q_pos, out_dtype=torch.float32,
                                prior=(m, l, o))
    assert (o2 - outs[0][0]).abs().max().item() <= 1e-5
    assert (l2 - outs[0][1]).abs().max().item() <= 1e-5
    ws = ops.WORKSPACES.get(torch.device(dev), 4096)
    torch.cuda.synchronize()
    assert torch.count_nonzero(ws[:4096]).item() == 0
    assert L.device_error() == 0


@pytest.mark.parametrize("D,H,H_kv", [(64, 64, 8), (96, 32, 2)])
def test_decode_dynamic_schedule_shapes(cuda_device, D, H, H_kv):
    """The dynamic schedule at other head dims and group counts (G = 8 and
    16, i.e. one q-head block per pair), with every batch row reading one
    shared K/V buffer (batch stride 0)."""
    ops = _ops()
    from halo_b200 import _lib as L
    g = torch.Generator().manual_seed(D + H)
    B, T, chunk = 2, 32768, 4096
    q = torch.randn(B, H, 1, D, generator=g).bfloat16()
    k1 = torch.randn(1, H_kv, T, D, generator=g).bfloat16()
    v1 = torch.randn(1, H_kv, T, D, generator=g).bfloat16()
    dev = cuda_device
    kd, vd = k1.to(dev).expand(B, -1, -1, -1), v1.to(dev).expand(B, -1, -1, -1)
    ch = [(kd[..., a:b, :], vd[..., a:b, :], a, False) for a, b in _bounds(T, chunk)]
    out, lse = ops.chunked_decode(q.to(dev), ch, out_dtype=torch.float32)
    st, sl = ops.chunked_decode(q.to(dev), ch, out_dtype=torch.float32, max_split_rows=2048)
    assert (out - st).abs().max().item() <= 1e-5 and (lse - sl).abs().max().item() <= 1e-5
    G = H // H_kv
    for hk in range(H_kv):
        hs = slice(hk * G, (hk + 1) * G)
        ro, rl = OA.full_attention_f64(q[:, hs], k1[:, hk:hk + 1].expand(B, -1, -1, -1),
                                       v1[:, hk:hk + 1].expand(B, -1, -1, -1))
        assert (out[:, hs].cpu().double() - ro[:, :, 0]).abs().max().item() <= OUT_TOL_16
        assert (lse[:, hs].cpu().double() - rl[:, :, 0]).abs().max().item() <= LSE_TOL
    assert L.device_error() == 0


def test_device_error_word_clear(cuda_device):
    from halo_b200 import _lib as L
    assert L.device_error(clear=True) == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [16, 32, 64, 80, 96, 128])
def test_decode_head_dims(cuda_device, dtype, D):
    """Every compiled head_dim (32/64/128-byte swizzle widths, 1..5 TMA
    boxes per row) against the fp64 oracle, with a ragged causal tail."""
    ops = _ops()
    g = torch.Generator().manual_seed(D)
    B, H, H_kv, T = 2, 8, 2, 777
    q = torch.randn(B, H, 1, D, generator=g).to(dtype)
    k = torch.randn(B, H_kv, T, D, generator=g).to(dtype)
    v = torch.randn(B, H_kv, T, D, generator=g).to(dtype)
    qp = torch.tensor([T - 1, 500], device=cuda_device)
    out, lse = ops.chunked_decode(q.to(cuda_device), _gpu_chunks(k, v, _bounds(T, 300), True),
                                  q_pos=qp, out_dtype=torch.float32)
    for b, p in enumerate((T - 1, 500)):
        ro, rl = OA.full_attention_f64(q[b:b + 1], k[b:b + 1], v[b:b + 1], q_pos=p)
        assert (out[b].cpu().double() - ro[0, :, 0]).abs().max().item() <= _tol(dtype)
        assert (lse[b].cpu().double() - rl[0, :, 0]).abs().max().item() <= LSE_TOL


def test_decode_without_lse_output(cuda_device):
    """``want_lse=False``: the output equals the one written alongside the
    log-sum-exp (same launches, the merge skips the lse store), with and
    without a prior running state, and ``None`` comes back for the lse."""
    ops = _ops()
    torch.manual_seed(3)
    B, H, H_kv, D, T = 2, 16, 4, 128, 3000
    q = torch.randn(B, H, 1, D, device=cuda_device).bfloat16()
    k = torch.randn(B, H_kv, T, D, device=cuda_device).bfloat16()
    v = torch.randn(B, H_kv, T, D, device=cuda_device).bfloat16()
    chunks = [(k[..., a:b, :], v[..., a:b, :], a, False) for a, b in _bounds(T, 1024)]
    ref_o, _ = OA.full_attention_f64(q.cpu(), k.cpu(), v.cpu())
    out_l, lse = ops.chunked_decode(q, chunks)
    out_n, none = ops.chunked_decode(q, chunks, want_lse=False)
    assert none is None and lse is not None
    assert torch.equal(out_l, out_n)
    assert (out_n.float().cpu().double() - ref_o[:, :, 0]).abs().max().item() <= OUT_TOL_16
    # a prior (m, l, o) from the first half folded into the second half
    m = torch.full((B, H), -float("inf"), device=cuda_device)
    l = torch.zeros(B, H, device=cuda_device)
    o = torch.zeros(B, H, D, device=cuda_device)
    ops.accumulate_decode(q, chunks[:2], m, l, o, scale=1.0 / math.sqrt(D), q_pos=None)
    out_p, none_p = ops.chunked_decode(q, chunks[2:], prior=(m, l, o), want_lse=False)
    assert none_p is None
    assert (out_p.float().cpu().double() - ref_o[:, :, 0]).abs().max().item() <= OUT_TOL_16
