"""GPU parity at the full shapes of the benchmarked workloads.

Each test runs the CUDA path through the same public entry point the
benchmark times, at the benchmark's shapes, and compares every KV-head
group with a float64 attention computed by torch on the GPU (``_f64_attend``
below: plain matmul / logsumexp, no library kernel of this package).  That
checker is itself pinned to the CPU oracle (``oracle.attention``) on a small
case in ``test_f64_checker_matches_oracle``; the full sizes are out of reach
of the CPU oracle in test time.  Selections come from the numpy oracle
(``oracle.scorer``) and KIVI codes from the plain-C oracle (``oracle/kivi_ref.c``).

Workloads (seeded N(0,1) synthetic data; keys of the decode-with-outliers
workloads get 4 seeded channels per KV head scaled by 10):

* 1M-token decode of one 64 q-head / 8 KV-head layer, head_dim 128, bf16,
  256 chunks of 4096, through ``ShardedDecoder`` on one GPU;
* chunked prefill: the first and the last 4096-query slice of a
  131072-token prompt (32 / 8 heads, head_dim 128, bf16, causal) against the
  accumulated keys, through ``ops.prefill_attention``;
* KIVI 2-bit decode: B4 x 65536 rows (65408 quantised, 128 fp16 recent),
  32 / 8 heads, group 32, through ``KIVICache``;
* tiered decode: one full layer, B8, 32 / 8 heads, 32 chunks of 1024,
  hot = chunk 0 + the 7 most recent, top-8 cold chunks per step, through
  ``TieredLayer.step``.

Tolerances: attention out <= 2e-3 max-abs (fp32 output of 16-bit inputs),
LSE <= 1e-4, selected chunks identical except exact score ties (relative gap
< 1e-6), KIVI codes / scale / zero bit-exact.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np
import pytest
import torch

from oracle import attention as OA
from oracle import scorer as OS

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OUT_TOL = 2e-3
LSE_TOL = 1e-4


def _f64_attend(q, k, v, *, scale, q_pos0=None, keep=None, q_block=256):
    """float64 attention of one KV head's query group on the GPU.

    ``q (B, G, T_q, D)``, ``k, v (B, T, D)``; query row ``i`` sits at
    position ``q_pos0 + i`` and sees keys ``j <= q_pos0 + i`` when
    ``q_pos0`` is given (causal), every key otherwise; ``keep (T,)`` bool
    restricts the keys further.  Returns ``out (B, G, T_q, D_v)`` and
    ``lse (B, G, T_q)`` in float64."""
    B, G, T_q, D = q.shape
    T = k.shape[-2]
    out = torch.empty(B, G, T_q, v.shape[-1], dtype=torch.float64, device=q.device)
    lse = torch.empty(B, G, T_q, dtype=torch.float64, device=q.device)
    pos = torch.arange(T, device=q.device)
    for b in range(B):
        kd = k[b].double()
        vd = v[b].double()
        for i0 in range(0, T_q, q_block):
            i1 = min(i0 + q_block, T_q)
            s = torch.matmul(q[b, :, i0:i1].double(), kd.T) * scale      # (G, tq, T)
            allowed = torch.ones(i1 - i0, T, dtype=torch.bool, device=q.device)
            if q_pos0 is not None:
                qp = torch.arange(i0, i1, device=q.device) + q_pos0
                allowed &= pos[None, :] <= qp[:, None]
            if keep is not None:
                allowed &= keep[None, :]
            s.masked_fill_(~allowed, float("-inf"))
            l = torch.logsumexp(s, dim=-1)
            w = torch.exp(s - l[..., None])
            w = torch.nan_to_num(w, nan=0.0)
            out[b, :, i0:i1] = torch.matmul(w, vd)
            lse[b, :, i0:i1] = l
            del s, w
    return out, lse


def _check_groups(out, lse, q, k, v, *, scale, q_pos0=None, keep=None, groups=None):
    """Compare ``out (B, H, T_q, D)`` / ``lse (B, H, T_q)`` with the float64
    checker one KV-head group at a time; returns the worst errors."""
    H, H_kv = q.shape[1], k.shape[1]
    G = H // H_kv
    worst_o = worst_l = 0.0
    for hk in (range(H_kv) if groups is None else groups):
        hs = slice(hk * G, (hk + 1) * G)
        ro, rl = _f64_attend(q[:, hs], k[:, hk], v[:, hk], scale=scale, q_pos0=q_pos0, keep=keep)
        eo = (out[:, hs].double() - ro).abs().max().item()
        el = (lse[:, hs].double() - rl).abs().max().item()
        worst_o, worst_l = max(worst_o, eo), max(worst_l, el)
        assert eo <= OUT_TOL, f"kv-head {hk}: out error {eo:.3e}"
        assert el <= LSE_TOL, f"kv-head {hk}: lse error {el:.3e}"
    return worst_o, worst_l


def _outliers(k, seed):
    """Scale 4 seeded channels of every KV head by 10."""
    g = torch.Generator().manual_seed(seed)
    for h in range(k.shape[1]):
        idx = torch.randperm(k.shape[-1], generator=g)[:4].to(k.device)
        k[:, h, :, idx] *= 10
    return k


def test_f64_checker_matches_oracle():
    """The GPU float64 checker equals the CPU oracle's float64 attention on
    a small case (decode, causal prefill with an offset, a key mask)."""
    g = torch.Generator().manual_seed(5)
    B, H, H_kv, D, T, T_q = 2, 8, 2, 64, 700, 37
    q = torch.randn(B, H, T_q, D, generator=g).bfloat16()
    k = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    v = torch.randn(B, H_kv, T, D, generator=g).bfloat16()
    keep = torch.rand(T, generator=g) > 0.3
    scale = 1 / math.sqrt(D)
    G = H // H_kv
    for q_pos0, kp in ((None, None), (T - T_q, None), (300, keep)):
        ro, rl = OA.full_attention_f64(q, k, v, scale=scale, keep=kp,
                                       q_pos=None if q_pos0 is None else q_pos0)
        for hk in range(H_kv):
            hs = slice(hk * G, (hk + 1) * G)
            go, gl = _f64_attend(q[:, hs].to(DEV), k[:, hk].to(DEV), v[:, hk].to(DEV), scale=scale,
                                 q_pos0=q_pos0, keep=None if kp is None else kp.to(DEV), q_block=16)
            assert (go.cpu() - ro[:, hs]).abs().max().item() <= 1e-12
            fin = torch.isfinite(rl[:, hs])
            assert torch.equal(torch.isfinite(gl.cpu()), fin)
            assert (gl.cpu()[fin] - rl[:, hs][fin]).abs().max().item() <= 1e-12


def test_cfg5_decode_full_million_tokens():
    """The 1M-token decode (B1, 64/8 heads, head_dim 128, bf16, 256 chunks
    of 4096) through ShardedDecoder on one GPU, called twice (the dynamic
    schedule may fold in another order each call), every KV-head group
    checked."""
    from halo_b200 import _lib as L
    from halo_b200.sharded import ShardedDecoder
    B, H, H_kv, D, T, C = 1, 64, 8, 128, 1 << 20, 4096
    g = torch.Generator(device=DEV).manual_seed(1000)
    k = torch.randn(B, H_kv, T, D, device=DEV, dtype=torch.bfloat16, generator=g)
    v = torch.randn(B, H_kv, T, D, device=DEV, dtype=torch.bfloat16, generator=g)
    q = torch.randn(B, H, D, device=DEV, dtype=torch.bfloat16,
                    generator=torch.Generator(device=DEV).manual_seed(7))
    dec = ShardedDecoder(k, v, start=0, chunk_size=C)
    assert len(dec.chunks) == 256
    scale = 1 / math.sqrt(D)
    results = []
    for _ in range(2):
        out = torch.full((B, H, D), float("nan"), device=DEV)
        lse = torch.full((B, H), float("nan"), device=DEV)
        dec(q, out=out, lse=lse)
        torch.cuda.synchronize()
        _check_groups(out[:, :, None], lse[:, :, None], q[:, :, None], k, v, scale=scale)
        results.append(out)
    assert (results[0] - results[1]).abs().max().item() <= 1e-5
    # the bf16 output the benchmark keeps is that result rounded once
    ob = torch.empty(B, H, D, device=DEV, dtype=torch.bfloat16)
    dec(q, out=ob, lse=torch.empty(B, H, device=DEV))
    assert (ob.float() - results[0]).abs().max().item() <= 2 ** -8 * results[0].abs().max().item() + 1e-5
    dec.close()
    assert L.device_error() == 0


def _cfg3_inputs(T=131072, H=32, H_kv=8, D=128):
    g = torch.Generator(device=DEV).manual_seed(3)
    k = torch.randn(1, H_kv, T, D, device=DEV, generator=g)
    v = torch.randn(1, H_kv, T, D, device=DEV, generator=g, dtype=torch.bfloat16)
    k = _outliers(k, 33).bfloat16()
    return k, v


@pytest.mark.parametrize("slice_index", [0, 31])
def test_cfg3_prefill_slice_full_size(slice_index):
    """One 4096-query slice of the 131072-token prompt (32/8 heads, head_dim
    128, bf16, keys with outlier channels) against every key it may see,
    called the way the chunked-prefill loop calls it; the last slice attends
    131072 keys, the first only its own causal triangle."""
    from halo_b200 import _lib as L
    from halo_b200 import ops
    H, H_kv, D, T, S = 32, 8, 128, 131072, 4096
    k, v = _cfg3_inputs(T, H, H_kv, D)
    s0 = slice_index * S
    q = torch.randn(1, H, S, D, device=DEV, dtype=torch.bfloat16,
                    generator=torch.Generator(device=DEV).manual_seed(300 + slice_index))
    kk, vv = k[..., :s0 + S, :], v[..., :s0 + S, :]
    out, lse = ops.prefill_attention(q, [(kk, vv, 0, True)], query_pos_offset=s0,
                                     out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert L.device_error() == 0
    _check_groups(out, lse, q, kk, vv, scale=1 / math.sqrt(D), q_pos0=s0)


@pytest.fixture(scope="module")
def c_oracle():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_build", "liboracle_kivi.so"))
    lib.oracle_kivi_quantize.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p]
    return lib


def _bits16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def test_cfg4_kivi_decode_full_size(c_oracle):
    """KIVI 2-bit decode at B4 x 65536 (65408 quantised rows + 128 fp16
    recent rows), 32/8 heads, head_dim 128, group 32, keys with outlier
    channels: codes, scales and zeros of the whole prefix bit-exact against
    the C oracle; out and LSE of the fused decode plus the recent fold
    against float64 attention over the reference's dequantised values."""
    from halo_b200 import _lib as L
    from halo_b200 import ops
    from halo_b200.baselines.kivi_cache import KIVICache, kivi_decode, unpack_codes
    B, H, H_kv, D, T, R = 4, 32, 8, 128, 65536, 128
    g = torch.Generator(device=DEV).manual_seed(4)
    k = torch.randn(B, H_kv, T, D, device=DEV, generator=g)
    v = torch.randn(B, H_kv, T, D, device=DEV, generator=g)
    q = torch.randn(B, H, 1, D, device=DEV, generator=g).half()
    k = _outliers(k, 44).half()
    v = v.half()
    cache = KIVICache(bits=2, group_size=32, residual_length=R, fused_attention=True)
    cache.update(k, v, layer_idx=0)
    kq, vq = cache._k_quant[0], cache._v_quant[0]
    Tq = T - R
    assert kq.T == Tq and cache._k_recent[0].shape[-2] == R

    # codes / scale / zero of the whole quantised prefix vs the C oracle
    deq = []
    for x, pk in ((k, kq), (v, vq)):
        rows = B * H_kv * Tq
        xb = x[:, :, :Tq].contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        ref_c = np.empty(rows * D, dtype=np.int8)
        ref_s = np.empty(rows * (D // 32), dtype=np.uint16)
        ref_z = np.empty_like(ref_s)
        c_oracle.oracle_kivi_quantize(xb.ctypes.data, rows, D, 32, 2, 0, ref_c.ctypes.data,
                                      ref_s.ctypes.data, ref_z.ctypes.data)
        got_c = unpack_codes(pk.codes[:, :, :Tq], 2).cpu().numpy().reshape(-1)
        assert np.array_equal(got_c.astype(np.int8), ref_c)
        assert np.array_equal(_bits16(pk.scale[:, :, :Tq]).reshape(-1), ref_s)
        assert np.array_equal(_bits16(pk.zero[:, :, :Tq]).reshape(-1), ref_z)
        # the reference's dequantisation (fp32 multiply, then add, then one
        # rounding to fp16) from the oracle's codes, as plain torch ops
        c = torch.from_numpy(ref_c).to(DEV).view(B, H_kv, Tq, D // 32, 32).float()
        s = torch.from_numpy(ref_s.view(np.float16)).to(DEV).view(B, H_kv, Tq, D // 32, 1).float()
        z = torch.from_numpy(ref_z.view(np.float16)).to(DEV).view(B, H_kv, Tq, D // 32, 1).float()
        deq.append((c * s + z).half().view(B, H_kv, Tq, D))
        del c, s, z
    kd = torch.cat([deq[0], cache._k_recent[0]], dim=-2)
    vd = torch.cat([deq[1], cache._v_recent[0]], dim=-2)
    del deq

    # the decode step as KIVICache.compute_attention runs it, kept in fp32
    q3 = q.squeeze(2).contiguous()
    scale = 1 / math.sqrt(D)
    o32 = torch.empty(B, H, D, device=DEV)
    l32 = torch.empty(B, H, device=DEV)
    kivi_decode(q3, kq, vq, Tq, 2, scale=scale, out=o32, lse=l32)
    ones = torch.ones(B, H, device=DEV)
    out, lse = ops.chunked_decode(q3, [(cache._k_recent[0], cache._v_recent[0], Tq, False)],
                                  scale=scale, prior=(l32, ones, o32), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert L.device_error() == 0
    _check_groups(out[:, :, None], lse[:, :, None], q, kd, vd, scale=scale)
    # the public call returns that result rounded once to fp16
    o16 = cache.compute_attention(q, layer_idx=0)
    assert o16.dtype == torch.float16 and o16.shape == (B, H, 1, D)
    assert (o16[:, :, 0].float() - out).abs().max().item() <= 2 ** -11 * out.abs().max().item() + 1e-5


def test_cfg2_tiered_layer_full_size():
    """One full layer of the tiered decode (B8, 32/8 heads, head_dim 128,
    bf16, 32 chunks of 1024, hot = chunk 0 + the 7 most recent, 24 cold
    chunks in pinned host memory, top-8 per step): per step the selection
    equals the numpy oracle's Quest top-k (modulo exact ties) and out/LSE
    equal float64 attention over the hot and selected chunks; the second
    step copies only the chunks that were not resident."""
    from halo_b200 import _lib as L
    from halo_b200.tiered import TieredLayer
    B, H, H_kv, D, C, P, k_sel = 8, 32, 8, 128, 1024, 32, 8
    hot = [0] + list(range(25, 32))
    g = torch.Generator(device=DEV).manual_seed(2)
    k = _outliers(torch.randn(B, H_kv, P * C, D, device=DEV, generator=g), 200).bfloat16()
    v = torch.randn(B, H_kv, P * C, D, device=DEV, generator=g, dtype=torch.bfloat16)
    lay = TieredLayer(k, v, chunk_size=C, hot_chunks=hot, n_slots=k_sel)
    kmin, kmax = OS.page_summaries(k.float().cpu().numpy(), C)
    gq = torch.Generator(device=DEV).manual_seed(22)
    prev = set()
    for _ in range(2):
        q = torch.randn(B, H, D, device=DEV, dtype=torch.bfloat16, generator=gq)
        n_before = lay.stats["refetched_chunks"]
        out = torch.empty(B, H, D, device=DEV)
        lse = torch.empty(B, H, device=DEV)
        out, lse, chosen = lay.step(q, k_sel=k_sel, out=out, lse=lse)
        torch.cuda.synchronize()
        qg = OS.gqa_mean_query(q.float().cpu().numpy()[:, :, None, :], H_kv, dtype="bf16")
        want, per_page = OS.select_topk(OS.score_pages(qg, kmin, kmax), k_sel, exclude=hot)
        want = [int(i) for i in want]
        if sorted(chosen) != sorted(want):
            kth = min(per_page[i] for i in want)
            for i in set(chosen) ^ set(want):
                assert abs(per_page[i] - kth) / max(abs(kth), 1e-30) < 1e-6
        assert not set(chosen) & set(hot)
        assert lay.stats["refetched_chunks"] - n_before == len(set(chosen) - prev)
        prev = set(chosen)
        keep = torch.zeros(P * C, dtype=torch.bool, device=DEV)
        for c in hot + chosen:
            keep[c * C:(c + 1) * C] = True
        _check_groups(out[:, :, None], lse[:, :, None], q[:, :, None], k, v,
                      scale=1 / math.sqrt(D), keep=keep)
    assert L.device_error() == 0
