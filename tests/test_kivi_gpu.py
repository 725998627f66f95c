"""GPU parity of the KIVI kernels: quantise / dequantise bit-exact with the
reference (golden vectors and the C oracle), fused 2/4/8-bit dequant-and-
attend decode vs the oracle's attention over the dequantised values (out
within 2e-3, LSE within 1e-4), and the reference's KIVICache tests."""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np
import pytest
import torch

import inputs as I
from oracle import attention as OA
from oracle import kivi as OK

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bits16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _assert_bits_equal_nan_aware(got_bits, want_bits, dtype):
    """Bit-exact, except that any NaN equals any NaN: x86 torch makes
    0 * inf a negative quiet NaN, CUDA the canonical positive one."""
    def isnan(b):
        if dtype == torch.float16:
            return ((b & 0x7C00) == 0x7C00) & ((b & 0x03FF) != 0)
        return ((b & 0x7F80) == 0x7F80) & ((b & 0x007F) != 0)
    nan_g, nan_w = isnan(got_bits), isnan(want_bits)
    np.testing.assert_array_equal(nan_g, nan_w)
    np.testing.assert_array_equal(got_bits[~nan_g], want_bits[~nan_w])


@pytest.mark.parametrize("name", list(I.KIVI_CASES))
def test_quantize_matches_reference_golden(name):
    from halo_b200.baselines.kivi_cache import _dequantize_per_group, _quantize_per_group
    g = I.load("kivi.npz")[name]
    x, bits = I.kivi_inputs(name)
    q, s, z = _quantize_per_group(x.to(DEV), bits=bits, group_size=32, axis=-1)
    np.testing.assert_array_equal(q.cpu().numpy(), g["codes"])
    np.testing.assert_array_equal(_bits16(s), g["scale_bits"])
    np.testing.assert_array_equal(_bits16(z), g["zero_bits"])
    dq = _dequantize_per_group(q, s, z, group_size=32)
    _assert_bits_equal_nan_aware(_bits16(dq), g["dq_bits"], x.dtype)


@pytest.fixture(scope="module")
def c_oracle():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_build", "liboracle_kivi.so"))
    lib.oracle_kivi_quantize.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p]
    return lib


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bits", [2, 4, 8])
def test_packed_quantize_matches_c_oracle(c_oracle, dtype, bits):
    from halo_b200.baselines.kivi_cache import quantize_packed
    g = torch.Generator().manual_seed(bits)
    x = torch.randn(2, 3, 777, 128, generator=g) * torch.rand(2, 3, 777, 1, generator=g) * 4
    x[..., 5] *= 10
    x = x.to(dtype)
    codes, scale, zero = quantize_packed(x.to(DEV), bits=bits, group_size=32)
    rows = x.numel() // 128
    ref_c = np.empty(rows * 128, dtype=np.int8)
    ref_s = np.empty(rows * 4, dtype=np.uint16)
    ref_z = np.empty_like(ref_s)
    xb = x.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    c_oracle.oracle_kivi_quantize(xb.ctypes.data, rows, 128, 32, bits, 0 if dtype == torch.float16 else 1,
                                  ref_c.ctypes.data, ref_s.ctypes.data, ref_z.ctypes.data)
    from halo_b200.baselines.kivi_cache import unpack_codes
    unpacked = unpack_codes(codes, bits).cpu().numpy().reshape(rows, 128)
    np.testing.assert_array_equal(unpacked.astype(np.int8), ref_c.reshape(rows, 128))
    if bits == 2:   # the device layout is the oracle's packing
        ref_packed = OK.pack_codes_2bit(ref_c.reshape(rows, 4, 32))
        np.testing.assert_array_equal(codes.cpu().numpy().reshape(rows, 32), ref_packed)
    np.testing.assert_array_equal(_bits16(scale).reshape(-1), ref_s)
    np.testing.assert_array_equal(_bits16(zero).reshape(-1), ref_z)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bits,D", [(2, 128), (2, 64), (4, 128), (8, 64)])
def test_fused_kivi_decode_matches_oracle(dtype, bits, D):
    from halo_b200.baselines.kivi_cache import _Packed, kivi_decode
    g = torch.Generator().manual_seed(100 + bits + D)
    B, H, H_kv, T = 2, 16, 4, 1000
    k = torch.randn(B, H_kv, T, D, generator=g)
    k[..., 3] *= 10
    v = torch.randn(B, H_kv, T, D, generator=g)
    q = torch.randn(B, H, D, generator=g).to(dtype)
    kq = _Packed(B, H_kv, D, dtype, torch.device(DEV), bits, 32)
    vq = _Packed(B, H_kv, D, dtype, torch.device(DEV), bits, 32)
    kq.append(k.to(dtype).to(DEV))
    vq.append(v.to(dtype).to(DEV))
    out, lse = kivi_decode(q.to(DEV), kq, vq, T, bits, scale=1 / math.sqrt(D),
                           out=torch.empty(B, H, D, device=DEV))
    kd = kq.dequantized().cpu()
    vd = vq.dequantized().cpu()
    # the dequantised values are the reference's (bit-exact checked above)
    ck, sk, zk = OK.quantize_per_group(k.to(dtype).float().numpy(), bits=bits, group_size=32,
                                       dtype="f16" if dtype == torch.float16 else "bf16",
                                       unsigned_codes=True)
    ref_kd = OK.dequantize_per_group(ck, sk, zk, dtype="f16" if dtype == torch.float16 else "bf16")
    np.testing.assert_array_equal(kd.float().numpy(), ref_kd)
    ro, rl = OA.full_attention_f64(q.unsqueeze(2), kd, vd)
    assert (out.cpu().double() - ro[:, :, 0]).abs().max().item() <= 2e-3
    assert (lse.cpu().double() - rl[:, :, 0]).abs().max().item() <= 1e-4


@pytest.mark.parametrize("G", [1, 8, 16])
def test_fused_kivi_decode_gqa_groups(G):
    """Both tile layouts of the fused kernel: groups of at most 8 q-heads use
    the transposed (keys-as-rows) MMA form, larger groups the q-heads-as-rows
    form."""
    from halo_b200.baselines.kivi_cache import _Packed, kivi_decode
    dtype, bits, D = torch.float16, 2, 128
    g = torch.Generator().manual_seed(200 + G)
    B, H_kv, T = 2, 2, 1500
    H = H_kv * G
    k = torch.randn(B, H_kv, T, D, generator=g)
    k[..., 5] *= 10
    v = torch.randn(B, H_kv, T, D, generator=g)
    q = torch.randn(B, H, D, generator=g).to(dtype)
    kq = _Packed(B, H_kv, D, dtype, torch.device(DEV), bits, 32)
    vq = _Packed(B, H_kv, D, dtype, torch.device(DEV), bits, 32)
    kq.append(k.to(dtype).to(DEV))
    vq.append(v.to(dtype).to(DEV))
    out, lse = kivi_decode(q.to(DEV), kq, vq, T, bits, scale=1 / math.sqrt(D),
                           out=torch.empty(B, H, D, device=DEV))
    ro, rl = OA.full_attention_f64(q.unsqueeze(2), kq.dequantized().cpu(), vq.dequantized().cpu())
    assert (out.cpu().double() - ro[:, :, 0]).abs().max().item() <= 2e-3
    assert (lse.cpu().double() - rl[:, :, 0]).abs().max().item() <= 1e-4


def test_kivi_cache_reference_behaviour():
    """Reference tests/test_kivi_cache.py:37-107 on the GPU cache."""
    from halo_b200.baselines.kivi_cache import KIVICache
    torch.manual_seed(0)
    c = KIVICache(bits=4, group_size=32, residual_length=32)
    K, V = c.update(torch.randn(1, 4, 100, 128, device=DEV).half(),
                    torch.randn(1, 4, 100, 128, device=DEV).half(), layer_idx=0)
    assert K.shape == (1, 4, 100, 128) and V.shape == (1, 4, 100, 128)
    K, V = c.update(torch.randn(1, 4, 10, 128, device=DEV).half(),
                    torch.randn(1, 4, 10, 128, device=DEV).half(), layer_idx=0)
    assert K.shape == (1, 4, 110, 128) and c.get_seq_length(0) == 110
    c = KIVICache(bits=2, group_size=32, residual_length=64)
    kf = torch.randn(1, 4, 200, 128, device=DEV).half()
    vf = torch.randn(1, 4, 200, 128, device=DEV).half()
    c.update(kf[..., :100, :], vf[..., :100, :], layer_idx=0)
    K, V = c.update(kf[..., 100:, :], vf[..., 100:, :], layer_idx=0)
    assert torch.equal(K[..., -64:, :], kf[..., -64:, :])
    assert torch.equal(V[..., -64:, :], vf[..., -64:, :])
    c = KIVICache(bits=2, group_size=32, residual_length=32)
    kf = torch.randn(1, 4, 96, 64, device=DEV).half()
    K, _ = c.update(kf, torch.randn(1, 4, 96, 64, device=DEV).half(), layer_idx=0)
    err = (K[..., :64, :] - kf[..., :64, :]).abs().float().mean().item()
    assert 1e-3 < err < 1.0
    assert KIVICache.from_memory_ratio(memory_ratio=4).bits == 4
    assert KIVICache.from_memory_ratio(memory_ratio=8).bits == 2
    assert KIVICache.from_memory_ratio(memory_ratio=2).bits == 8


def test_kivi_cache_fused_attention_matches_dequantised_attention():
    from halo_b200.baselines.kivi_cache import KIVICache
    torch.manual_seed(1)
    B, H, H_kv, D = 2, 16, 4, 128
    c = KIVICache(bits=2, group_size=32, residual_length=128, fused_attention=True)
    full = KIVICache(bits=2, group_size=32, residual_length=128, fused_attention=False)
    k = torch.randn(B, H_kv, 3000, D, device=DEV).half()
    v = torch.randn(B, H_kv, 3000, D, device=DEV).half()
    for a, b in ((0, 2900), (2900, 2950), (2950, 3000)):
        c.update(k[..., a:b, :], v[..., a:b, :], layer_idx=0)
        Kd, Vd = full.update(k[..., a:b, :], v[..., a:b, :], layer_idx=0)
    q = torch.randn(B, H, 1, D, device=DEV).half()
    out = c.compute_attention(q, layer_idx=0)
    ro, _ = OA.full_attention_f64(q.cpu(), Kd.cpu(), Vd.cpu())
    assert (out.float().cpu() - ro.float()).abs().max().item() <= 2e-3 + 1e-3  # fp16 output rounding


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_kivi_cache_fused_decode_loop_tracks_updates(dtype):
    """A decode loop on two layers: one-row updates, with the fused
    attention after every one.  The updates cross quantisation boundaries
    (the recent rows and the packed prefix change) and outgrow the packed
    storage's first capacity, and some calls run on a side stream; each
    output must match attention over the unfused cache's dequantised K/V
    (2e-3, plus half a unit in the last place of the output dtype)."""
    from halo_b200.baselines.kivi_cache import KIVICache
    torch.manual_seed(5)
    B, H, H_kv, D, steps = 2, 8, 2, 128, 260
    c = KIVICache(bits=2, group_size=32, residual_length=128, fused_attention=True)
    full = KIVICache(bits=2, group_size=32, residual_length=128, fused_attention=False)
    k = torch.randn(2, B, H_kv, 200 + steps, D, device=DEV).to(dtype)
    v = torch.randn(2, B, H_kv, 200 + steps, D, device=DEV).to(dtype)
    half_ulp = 2.0 ** -11 if dtype == torch.float16 else 2.0 ** -8
    side = torch.cuda.Stream()
    caps = set()
    for t in range(steps + 1):
        a, b = (0, 200) if t == 0 else (199 + t, 200 + t)
        for layer in range(2):
            c.update(k[layer, ..., a:b, :], v[layer, ..., a:b, :], layer_idx=layer)
            Kd, Vd = full.update(k[layer, ..., a:b, :], v[layer, ..., a:b, :], layer_idx=layer)
            q = torch.randn(B, H, 1, D, device=DEV).to(dtype)
            if t % 7 == 3:
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    out = c.compute_attention(q, layer_idx=layer)
                torch.cuda.current_stream().wait_stream(side)
            else:
                out = c.compute_attention(q, layer_idx=layer)
            if t % 13 == 0 or t == steps:
                ro, _ = OA.full_attention_f64(q.cpu(), Kd.cpu(), Vd.cpu())
                err = (out.cpu().double() - ro).abs().max().item()
                tol = 2e-3 + half_ulp * max(1.0, ro.abs().max().item())
                assert err <= tol, (t, layer, err, tol)
        caps.add(c._k_quant[0].codes.shape[2])
    assert len(caps) >= 2, "the packed storage never grew"
    assert c.get_seq_length(0) == 200 + steps


def test_kivi_cache_fused_decode_without_recent_rows():
    """residual_length 0 and a multiple of the group size: every row is
    quantised and the fused call returns the packed prefix's attention
    alone.  Two calls in a row: the first result must not change when the
    second call reuses the cache's fp32 state buffers."""
    from halo_b200.baselines.kivi_cache import KIVICache
    torch.manual_seed(6)
    B, H, H_kv, D = 2, 8, 2, 128
    c = KIVICache(bits=2, group_size=32, residual_length=0, fused_attention=True)
    full = KIVICache(bits=2, group_size=32, residual_length=0, fused_attention=False)
    k = torch.randn(B, H_kv, 512, D, device=DEV).half()
    v = torch.randn(B, H_kv, 512, D, device=DEV).half()
    c.update(k, v, layer_idx=0)
    Kd, Vd = full.update(k, v, layer_idx=0)
    assert c._k_recent[0].shape[-2] == 0
    q1 = torch.randn(B, H, 1, D, device=DEV).half()
    q2 = torch.randn(B, H, 1, D, device=DEV).half()
    out1 = c.compute_attention(q1, layer_idx=0)
    keep = out1.clone()
    out2 = c.compute_attention(q2, layer_idx=0)
    torch.cuda.synchronize()
    assert torch.equal(out1, keep)
    for q, out in ((q1, out1), (q2, out2)):
        ro, _ = OA.full_attention_f64(q.cpu(), Kd.cpu(), Vd.cpu())
        assert (out.float().cpu() - ro.float()).abs().max().item() <= 2e-3 + 1e-3
