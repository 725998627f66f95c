"""GPU parity of the tensor-core chunked-prefill kernel (halo_prefill_attention)
against the reference's golden vectors and the float64 oracle.  Contract:
fp32 output within 2e-3 max-abs, LSE within 1e-4 (natural log), rows with no
visible key give zeros and -inf, running-state folds equal one call."""
from __future__ import annotations


import pytest
import torch

import inputs as I
from oracle import attention as OA

pytestmark = pytest.mark.gpu
DEV = "cuda"
OUT_TOL = 2e-3
LSE_TOL = 1e-4


def _ops():
    from halo_b200 import ops
    return ops


def _outliers(k, seed):
    g = torch.Generator().manual_seed(seed)
    for h in range(k.shape[1]):
        k[:, h, :, torch.randperm(k.shape[-1], generator=g)[:4]] *= 10
    return k


def _qkv(B, H, H_kv, T, T_q, D, dtype, seed, outliers=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, T_q, D, generator=g)
    k = torch.randn(B, H_kv, T, D, generator=g)
    v = torch.randn(B, H_kv, T, D, generator=g)
    if outliers:
        k = _outliers(k, seed + 1)
    return q.to(dtype), k.to(dtype), v.to(dtype)


def _check(out, lse, ro, rl):
    fin = torch.isfinite(rl)
    assert (out.cpu().double() - ro).abs().max().item() <= OUT_TOL
    assert torch.equal(torch.isneginf(lse.cpu()), torch.isneginf(rl))
    assert (lse.cpu().double()[fin] - rl[fin]).abs().max().item() <= LSE_TOL


@pytest.mark.parametrize("name", [n for n in I.PREFILL_CASES if "f32" not in n])
def test_prefill_kernel_matches_reference_golden(name):
    ops = _ops()
    (q, k, v), T_cold, chunk = I.prefill_inputs(name)
    g = I.load("attention.npz")[name]
    T, T_q = k.shape[-2], q.shape[-2]
    kd, vd = k.to(DEV), v.to(DEV)
    chunks = [(kd[..., a:min(a + chunk, T), :], vd[..., a:min(a + chunk, T), :], a, True)
              for a in range(0, T, chunk)]
    assert ops.prefill_supported(q, chunks)
    out, lse = ops.prefill_attention(q.to(DEV), chunks, query_pos_offset=T - T_q,
                                     out_dtype=torch.float32)
    assert (out.cpu() - torch.from_numpy(g["out"])).abs().max().item() <= OUT_TOL
    assert (lse.cpu() - torch.from_numpy(g["lse"])).abs().max().item() <= LSE_TOL


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("T_q,T_hist,G", [(1, 300, 4), (77, 0, 1), (128, 128, 4), (300, 1000, 4),
                                          (513, 2048, 2)])
def test_prefill_causal_matches_oracle(dtype, D, T_q, T_hist, G):
    """A slice of T_q queries after T_hist cached rows, causal over all."""
    ops = _ops()
    B, H_kv = 2, 2
    H = H_kv * G
    T = T_hist + T_q
    q, k, v = _qkv(B, H, H_kv, T, T_q, D, dtype, seed=T_q * 7 + T_hist + D)
    kd, vd = k.to(DEV), v.to(DEV)
    chunks = [(kd[..., a:min(a + 512, T), :], vd[..., a:min(a + 512, T), :], a, True)
              for a in range(0, T, 512)]
    out, lse = ops.prefill_attention(q.to(DEV), chunks, query_pos_offset=T_hist,
                                     out_dtype=torch.float32)
    ro, rl = OA.full_attention_f64(q, k, v, q_pos=T_hist)
    _check(out, lse, ro, rl)
    # the output in the input dtype is the fp32 result rounded once
    out_q, _ = ops.prefill_attention(q.to(DEV), chunks, query_pos_offset=T_hist)
    assert out_q.dtype == dtype
    assert torch.equal(out_q.cpu(), out.cpu().to(dtype))


def test_prefill_scattered_chunks_strides_and_noncausal_mix():
    """Chunks from separate allocations (one strided view, one batch-
    broadcast-free copy), a non-causal chunk, and queries at an offset that
    hides part of the last causal chunk."""
    ops = _ops()
    B, H, H_kv, D, T_q = 2, 8, 2, 128, 200
    q, k, v = _qkv(B, H, H_kv, 1500, T_q, D, torch.bfloat16, seed=5)
    # chunk 0: a (B, T, H_kv, D) layout viewed as (B, H_kv, T, D)
    k0 = k[..., :700, :].transpose(1, 2).contiguous().to(DEV).transpose(1, 2)
    v0 = v[..., :700, :].transpose(1, 2).contiguous().to(DEV).transpose(1, 2)
    k1, v1 = k[..., 700:1100, :].to(DEV), v[..., 700:1100, :].to(DEV)
    k2, v2 = k[..., 1100:, :].to(DEV), v[..., 1100:, :].to(DEV)
    q_off = 1200     # keys 1200+i .. visible to query i; rows 1401.. hidden from early queries
    chunks = [(k0, v0, 0, False), (k1, v1, 700, True), (k2, v2, 1100, True)]
    out, lse = ops.prefill_attention(q.to(DEV), chunks, query_pos_offset=q_off,
                                     out_dtype=torch.float32)
    # reference: causal over all keys at q_off (chunk 0 entirely before every query)
    ro, rl = OA.full_attention_f64(q, k, v, q_pos=q_off)
    _check(out, lse, ro, rl)


def test_prefill_rows_without_visible_keys():
    """Queries positioned before every causal key: zeros and -inf; a prior
    state passes through unchanged in value."""
    ops = _ops()
    B, H, H_kv, D, T_q = 1, 4, 4, 64, 130
    q, k, v = _qkv(B, H, H_kv, 300, T_q, D, torch.float16, seed=9)
    kd, vd = k.to(DEV), v.to(DEV)
    chunks = [(kd, vd, 1000, True)]                 # keys at 1000.. ; queries at 0..129
    out, lse = ops.prefill_attention(q.to(DEV), chunks, query_pos_offset=0,
                                     out_dtype=torch.float32)
    assert torch.count_nonzero(out).item() == 0
    assert torch.isneginf(lse).all().item()
    # half the rows see some keys: queries at 900.. see keys 1000..(900+i)
    out, lse = ops.prefill_attention(q.to(DEV), chunks, query_pos_offset=900,
                                     out_dtype=torch.float32)
    ro, rl = OA.full_attention_f64(q, k, v, q_pos=900 - 1000)
    _check(out, lse, ro, rl)


def test_prefill_running_state_folds_equal_one_call():
    ops = _ops()
    B, H, H_kv, D, T_q, T = 1, 8, 2, 128, 256, 2000
    q, k, v = _qkv(B, H, H_kv, T, T_q, D, torch.bfloat16, seed=21)
    kd, vd, qd = k.to(DEV), v.to(DEV), q.to(DEV)
    parts = [(0, 900), (900, 1500), (1500, T)]
    m = torch.full((B, H, T_q), float("-inf"), device=DEV)
    l = torch.zeros(B, H, T_q, device=DEV)
    o = torch.zeros(B, H, T_q, D, device=DEV)
    for a, b in parts[:2]:
        ops.prefill_attention(qd, [(kd[..., a:b, :], vd[..., a:b, :], a, True)],
                              query_pos_offset=T - T_q, state=(m, l, o), accumulate=True)
    a, b = parts[2]
    out, lse = ops.prefill_attention(qd, [(kd[..., a:b, :], vd[..., a:b, :], a, True)],
                                     query_pos_offset=T - T_q, state=(m, l, o),
                                     out_dtype=torch.float32)
    ro, rl = OA.full_attention_f64(q, k, v, q_pos=T - T_q)
    _check(out, lse, ro, rl)


def test_prefill_more_chunks_than_one_call_takes():
    """100 non-contiguous chunks (every other 32-row block of a buffer):
    the wrapper splits them over calls and carries the running state."""
    ops = _ops()
    B, H, H_kv, D, T_q = 1, 4, 1, 64, 64
    q, k, v = _qkv(B, H, H_kv, 6400, T_q, D, torch.bfloat16, seed=33)
    kd, vd = k.to(DEV), v.to(DEV)
    keep = torch.zeros(6400, dtype=torch.bool)
    chunks = []
    for c in range(0, 6400, 64):
        chunks.append((kd[..., c:c + 32, :], vd[..., c:c + 32, :], c, False))
        keep[c:c + 32] = True
    assert len(chunks) > ops.PREFILL_MAX_CHUNKS
    out, lse = ops.prefill_attention(q.to(DEV), chunks, query_pos_offset=6400,
                                     out_dtype=torch.float32)
    ro, rl = OA.full_attention_f64(q, k, v, keep=keep)
    _check(out, lse, ro, rl)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prefill_large_slice_outlier_keys(dtype):
    """A 1024-query slice after 7K rows of history, outlier keys: peaked
    softmax rows stress the P precision (bf16 hi + lo, fp16 single)."""
    ops = _ops()
    B, H, H_kv, D, T_q, T = 1, 8, 2, 128, 1024, 8192
    q, k, v = _qkv(B, H, H_kv, T, T_q, D, dtype, seed=77)
    kd, vd = k.to(DEV), v.to(DEV)
    chunks = [(kd[..., a:a + 4096, :], vd[..., a:a + 4096, :], a, True) for a in range(0, T, 4096)]
    out, lse = ops.prefill_attention(q.to(DEV), chunks, query_pos_offset=T - T_q,
                                     out_dtype=torch.float32)
    ro, rl = OA.full_attention_f64(q, k, v, q_pos=T - T_q)
    _check(out, lse, ro, rl)
    from halo_b200 import _lib as L
    assert L.device_error() == 0


def test_multi_query_attention_uses_prefill_kernel():
    from halo_b200 import _lib as L
    ops = _ops()
    q, k, v = _qkv(1, 4, 2, 600, 100, 128, torch.bfloat16, seed=3)
    chunks = [(k.to(DEV), v.to(DEV), 0, True)]
    n0 = L.launch_count()
    out, lse = ops.multi_query_attention(q.to(DEV), chunks, query_pos_offset=500,
                                         out_dtype=torch.float32)
    assert L.launch_count() - n0 == 2          # the fp16 copy of V + one kp3_kernel launch
    ro, rl = OA.full_attention_f64(q, k, v, q_pos=500)
    _check(out, lse, ro, rl)


def _f64_causal_gpu(q, k, v, q_pos):
    """Float64 causal attention on the GPU (query i sees keys <= q_pos + i)."""
    import math
    B, H, T_q, D = q.shape
    G = H // k.shape[1]
    kk = k.double().repeat_interleave(G, 1)
    vv = v.double().repeat_interleave(G, 1)
    s = (q.double() @ kk.transpose(-1, -2)) / math.sqrt(D)
    qi = torch.arange(T_q, device=q.device)[:, None] + q_pos
    kj = torch.arange(k.shape[-2], device=q.device)[None, :]
    s = s.masked_fill(kj > qi, float("-inf"))
    return torch.softmax(s, -1) @ vv, torch.logsumexp(s, -1)


@pytest.mark.parametrize("dtype,D", [(torch.bfloat16, 128), (torch.float16, 128),
                                     (torch.bfloat16, 64)])
def test_prefill_split_last_wave_units(dtype, D):
    """More query-tile units than SMs with a remainder: the lightest units of
    the last wave run as two half-walk CTAs whose partials a merge kernel
    folds; the result equals float64 attention like every other unit."""
    from halo_b200 import _lib as L
    ops = _ops()
    B, H, H_kv, T_q, T = 1, 32, 8, 2048, 4096
    units = (T_q // 256) * B * H
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    split = units > sms and units % sms != 0
    q, k, v = _qkv(B, H, H_kv, T, T_q, D, dtype, seed=91)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    chunks = [(kd[..., a:a + 1024, :], vd[..., a:a + 1024, :], a, True) for a in range(0, T, 1024)]
    n0 = L.launch_count()
    out, lse = ops.prefill_attention(qd, chunks, query_pos_offset=T - T_q,
                                     out_dtype=torch.float32)
    launches = L.launch_count() - n0
    # v16 copy (bf16 only) + kp3, + the merge when units were split
    assert launches == (1 if dtype == torch.bfloat16 else 0) + 1 + (1 if split else 0)
    ro, rl = _f64_causal_gpu(qd, kd, vd, T - T_q)
    assert (out.double() - ro).abs().max().item() <= OUT_TOL
    assert (lse.double() - rl).abs().max().item() <= LSE_TOL
    # a second call (workspace reused) gives the same result
    out2, lse2 = ops.prefill_attention(qd, chunks, query_pos_offset=T - T_q,
                                       out_dtype=torch.float32)
    assert torch.equal(out, out2) and torch.equal(lse, lse2)
    assert L.device_error() == 0
