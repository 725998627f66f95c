"""Pin the CPU oracle to golden vectors produced by the reference's own code.

The fixtures in ``tests/golden/*.npz`` were written by
``tests/golden/make_golden.py`` running the reference (lzbaclz/HALO) Python
implementation; inputs are regenerated from seeds and checked by digest.
"""
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
from oracle import scorer as OS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _check_digest(d, *ts):
    assert d["digest"].tobytes().decode() == I.digest(*ts), \
        "seeded inputs changed; regenerate tests/golden with make_golden.py"


def test_kivi_2bit_device_layout_known_answers():
    """16 codes per little-endian 32-bit word, code e at bit 16*(e & 1) +
    2*(e >> 1): even codes fill the low half, odd codes the high half, pair
    (2q, 2q+1) at bit 2q of each half.  Codes e % 4 put 0/2 in the low half
    (0x8888) and 1/3 in the high half (0xDDDD); codes (e % 16) // 4 give
    0, 0, 1, 1, 2, 2, 3, 3 in both halves (0xFA50)."""
    row = np.array([e % 4 for e in range(32)], dtype=np.int8).reshape(1, 32)
    np.testing.assert_array_equal(OK.pack_codes_2bit(row), [0x88, 0x88, 0xDD, 0xDD] * 2)
    row = np.array([(e % 16) // 4 for e in range(32)], dtype=np.int8).reshape(1, 32)
    np.testing.assert_array_equal(OK.pack_codes_2bit(row), [0x50, 0xFA, 0x50, 0xFA] * 2)
    rng = np.random.default_rng(0)
    c = rng.integers(0, 4, size=(3, 4, 32)).astype(np.int8)
    np.testing.assert_array_equal(OK.unpack_codes_2bit(OK.pack_codes_2bit(c), 32), c)


@pytest.fixture(scope="module")
def att():
    return I.load("attention.npz")


@pytest.mark.parametrize("name", list(I.WALK_CASES))
def test_oracle_walk_matches_reference(att, name):
    (q, k, v), chunk = I.walk_inputs(name)
    g = att[name]
    _check_digest(g, q, k, v)
    chunks = [(k[..., c0:c0 + chunk, :], v[..., c0:c0 + chunk, :], c0, False)
              for c0 in range(0, k.shape[-2], chunk)]
    o, l = OA.chunked_attention(q, chunks)
    np.testing.assert_allclose(o.numpy(), g["out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(l.numpy(), g["lse"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name", list(I.DECODE_CASES))
def test_oracle_compute_attention_decode(att, name):
    (q, k, v), T_cold, chunk = I.decode_inputs(name)
    g = att[name]
    _check_digest(g, q, k, v)
    o, l = OA.compute_attention(q, cold_k=k[..., :T_cold, :], cold_v=v[..., :T_cold, :],
                                gpu_k=k[..., T_cold:, :], gpu_v=v[..., T_cold:, :],
                                chunk_size=chunk)
    np.testing.assert_allclose(o.numpy(), g["out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(l.numpy(), g["lse"], rtol=1e-6, atol=1e-6)
    # the reference returns out.to(q.dtype); ours rounds the same fp32 value
    np.testing.assert_array_equal(o.to(q.dtype).float().numpy(), g["out_qdtype"])
    n = math.ceil(T_cold / chunk) + math.ceil((k.shape[-2] - T_cold) / chunk)
    assert n == int(g["n_chunks"])


@pytest.mark.parametrize("name", list(I.PREFILL_CASES))
def test_oracle_compute_attention_prefill_causal(att, name):
    (q, k, v), T_cold, chunk = I.prefill_inputs(name)
    g = att[name]
    _check_digest(g, q, k, v)
    o, l = OA.compute_attention(q, cold_k=k[..., :T_cold, :], cold_v=v[..., :T_cold, :],
                                gpu_k=k[..., T_cold:, :], gpu_v=v[..., T_cold:, :],
                                chunk_size=chunk)
    np.testing.assert_allclose(o.numpy(), g["out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(l.numpy(), g["lse"], rtol=1e-6, atol=1e-6)
    # reference out.to(q.dtype) may differ by one rounding step at most
    diff = (o.to(q.dtype).float() - torch.from_numpy(g["out_qdtype"])).abs().max().item()
    assert diff <= (1e-6 if q.dtype == torch.float32 else 1e-2)


def test_oracle_config1():
    g = I.load("config1.npz")["config1"]
    q, k, v = I.config1_inputs()
    _check_digest(g, q, k, v)
    order = [int(c) for c in g["order"]]
    chunks = [(k[..., c * 512:(c + 1) * 512, :], v[..., c * 512:(c + 1) * 512, :], c * 512, False)
              for c in order]
    o, l = OA.chunked_attention(q, chunks)
    np.testing.assert_allclose(o[:, :, 0].numpy(), g["out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(l[:, :, 0].numpy(), g["lse"], rtol=1e-6, atol=1e-6)
    # and the fp64 one-shot truth agrees within fp32 noise
    o64, l64 = OA.full_attention_f64(q, k, v)
    assert (o64[:, :, 0].float() - torch.from_numpy(g["out"])).abs().max() < 1e-5
    assert (l64[:, :, 0].float() - torch.from_numpy(g["lse"])).abs().max() < 1e-5


def test_oracle_acc_state_consistent():
    (q, k, v), chunk = I.walk_inputs("walk_f32_gqa4")
    chunks = [(k[..., c0:c0 + chunk, :], v[..., c0:c0 + chunk, :], c0, True)
              for c0 in range(0, k.shape[-2], chunk)]
    m, l, o = OA.acc_state_from_chunks(q, chunks, q_pos=150)
    out, lse = OA.chunked_attention(q, chunks, q_pos=150)
    torch.testing.assert_close(o / l.unsqueeze(-1), out, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(m + torch.log(l), lse, rtol=1e-6, atol=1e-6)


def _to_f32(t: torch.Tensor) -> np.ndarray:
    return t.float().numpy()


@pytest.mark.parametrize("name", list(I.KIVI_CASES))
def test_oracle_kivi_bit_exact(name):
    g = I.load("kivi.npz")[name]
    x, bits = I.kivi_inputs(name)
    _check_digest(g, x)
    dt = "f16" if x.dtype == torch.float16 else "bf16"
    codes, scale, zero = OK.quantize_per_group(_to_f32(x), bits=bits, group_size=32, dtype=dt)
    np.testing.assert_array_equal(codes, g["codes"])
    tdt = torch.float16 if dt == "f16" else torch.bfloat16
    sb = torch.from_numpy(scale).to(tdt).view(torch.int16).numpy().view(np.uint16)
    zb = torch.from_numpy(zero).to(tdt).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(sb, g["scale_bits"])
    np.testing.assert_array_equal(zb, g["zero_bits"])
    dq = OK.dequantize_per_group(codes, scale, zero, dtype=dt)
    dqb = torch.from_numpy(dq).to(tdt).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(dqb, g["dq_bits"])
    # 2-bit packing round trip
    if bits == 2:
        np.testing.assert_array_equal(OK.unpack_codes_2bit(OK.pack_codes_2bit(codes), 32), codes)


@pytest.fixture(scope="module")
def c_oracle():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_build", "liboracle_kivi.so"))
    lib.oracle_kivi_quantize.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p]
    lib.oracle_kivi_dequantize.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                           ctypes.c_void_p]
    return lib


@pytest.mark.parametrize("name", list(I.KIVI_CASES))
def test_c_oracle_kivi_bit_exact(c_oracle, name):
    g = I.load("kivi.npz")[name]
    x, bits = I.kivi_inputs(name)
    D = x.shape[-1]
    rows = x.numel() // D
    xb = x.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    codes = np.empty(rows * D, dtype=np.int8)
    sc = np.empty(rows * D // 32, dtype=np.uint16)
    ze = np.empty_like(sc)
    dt = 0 if x.dtype == torch.float16 else 1
    c_oracle.oracle_kivi_quantize(xb.ctypes.data, rows, D, 32, bits, dt, codes.ctypes.data,
                                  sc.ctypes.data, ze.ctypes.data)
    np.testing.assert_array_equal(codes, g["codes"].reshape(-1))
    np.testing.assert_array_equal(sc, g["scale_bits"].reshape(-1))
    np.testing.assert_array_equal(ze, g["zero_bits"].reshape(-1))
    dq = np.empty(rows * D, dtype=np.uint16)
    c_oracle.oracle_kivi_dequantize(codes.ctypes.data, sc.ctypes.data, ze.ctypes.data, rows, D, 32,
                                    dt, dq.ctypes.data)
    np.testing.assert_array_equal(dq, g["dq_bits"].reshape(-1))


@pytest.mark.parametrize("name", list(I.SCORER_CASES))
def test_oracle_scorer(name):
    g = I.load("scorer.npz")[name]
    K, q, page, mr, mp = I.scorer_inputs(name)
    _check_digest(g, K, q)
    dt = "bf16" if K.dtype == torch.bfloat16 else "f32"
    kmin, kmax = OS.page_summaries(_to_f32(K), page)
    if dt == "bf16":
        np.testing.assert_array_equal(OS.f32_to_bf16_bits(kmin), g["kmin_bits"])
        np.testing.assert_array_equal(OS.f32_to_bf16_bits(kmax), g["kmax_bits"])
    else:
        np.testing.assert_array_equal(kmin, g["kmin"])
        np.testing.assert_array_equal(kmax, g["kmax"])
    qg = OS.gqa_mean_query(_to_f32(q), K.shape[1], dtype=dt)
    scores = OS.score_pages(qg, kmin, kmax)
    np.testing.assert_allclose(scores, g["scores"], rtol=2e-6, atol=2e-5)
    kk = OS.num_hot_pages(scores.shape[-1], mr, mp)
    top, per_page = OS.select_topk(scores, kk)
    ref_top = g["topk"]
    assert len(top) == len(ref_top)
    if set(top.tolist()) != set(ref_top.tolist()):
        # only exact-score ties may flip: compare the selected score multisets
        ref_pp = g["scores"].max(axis=(0, 1, 2))
        np.testing.assert_allclose(np.sort(per_page[top]), np.sort(ref_pp[ref_top]), rtol=1e-6)


@pytest.mark.parametrize("name", list(I.PRESS_CASES))
def test_oracle_press_scorer(name):
    """HALOPress ablation scorer: page means bit-exact (bf16 / fp32), the
    closed-form score's top-k equal to the reference's selection."""
    g = I.load("press.npz")[name]
    K, q, cfg = I.press_inputs(name)
    assert g["digest"].item().decode() == I.digest(K, q)
    dt = "bf16" if K.dtype == torch.bfloat16 else "f32"
    km = OS.page_means(K.float().numpy(), cfg["page_size"], dtype=dt)
    ref = OS.bf16_bits_to_f32(g["kmean_bits"]) if dt == "bf16" else g["kmean"]
    np.testing.assert_array_equal(km, ref)
    qg = OS.gqa_mean_query(q.float().numpy(), K.shape[1], dtype=dt)
    sc = OS.press_scores(qg, km, alpha=cfg["halopress_alpha"], beta=cfg["halopress_beta"],
                         gamma=cfg["halopress_gamma"], sink_tokens=cfg["halopress_sink_tokens"],
                         refresh_window=cfg["halopress_refresh_window"],
                         page_size=cfg["page_size"])
    k = OS.num_hot_pages(sc.shape[0], cfg["memory_ratio"], cfg["min_pages_selected"])
    np.testing.assert_array_equal(OS.topk_sorted(sc, k), g["topk"])


@pytest.mark.parametrize("name", list(I.PRESS_CASES))
def test_host_ablation_scorers_match_reference(name):
    """The uniform-random and FIFO scorers are host index rules: identical
    selections to the reference's for the same seed and page count."""
    from halo_b200.baselines.scorer_ablations import (AblationScorerConfig, FIFOScorerAdapter,
                                                      UniformRandomScorerAdapter)
    g = I.load("press.npz")[name]
    K, q, cfg = I.press_inputs(name)
    c = AblationScorerConfig(**cfg)
    for cls, key in ((UniformRandomScorerAdapter, "uniform"), (FIFOScorerAdapter, "fifo")):
        ad = cls(c)
        ad.observe_keys(0, K)
        top = ad.select_hot_pages(0, q)
        np.testing.assert_array_equal(top.numpy(), g[key])
        assert ad.score_calls == 1 and ad.cumulative_hot_pages == len(g[key])
