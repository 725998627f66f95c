"""GPU tests of the drop-in API (``halo_b200`` mirrors ``halo``), ported from
the reference's own test scenarios (lzbaclz/HALO ``tests/``) and extended
with golden vectors through ``compute_attention`` with a real cold tier."""
from __future__ import annotations

import math
import os
import random

import pytest
import torch

import inputs as I
from oracle import attention as OA

pytestmark = pytest.mark.gpu
os.environ.setdefault("TRANSFORMERS_VERBOSITY", "error")
DEV = "cuda"


def _ref_attention(q, k, v):
    """Naive full attention (last query over all keys), fp32 -- the reference
    tests' ground truth (tests/test_kv_cache_chunked.py:20-32)."""
    H, H_kv = q.shape[1], k.shape[1]
    if H != H_kv:
        k = k.repeat_interleave(H // H_kv, dim=1)
        v = v.repeat_interleave(H // H_kv, dim=1)
    qk = torch.matmul(q.float(), k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    return torch.matmul(torch.softmax(qk, dim=-1), v.float())


def _make_qkv(B=1, H=4, H_kv=4, T=128, D=32, dtype=torch.float32, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(B, H, 1, D, generator=g, dtype=dtype).to(DEV),
            torch.randn(B, H_kv, T, D, generator=g, dtype=dtype).to(DEV),
            torch.randn(B, H_kv, T, D, generator=g, dtype=dtype).to(DEV))


def _cache(H_kv=2, D=32, chunk=64, hot_ratio=1.0, recent=64, dtype=torch.float32):
    from halo_b200 import (HALOCacheChunked, HALOConfig, HALODemoter, HALORefetcher,
                           HALOScorer, MemoryTier, TieredStorage)
    cfg = HALOConfig(hot_ratio=hot_ratio, tiers=("gpu", "dram"))
    st = TieredStorage(tiers=[MemoryTier.GPU, MemoryTier.DRAM], num_layers=1, num_kv_heads=H_kv,
                       head_dim=D, block_size=32, dtype=dtype, device=torch.device(DEV))
    return HALOCacheChunked(config=cfg, storage=st, scorer=HALOScorer(cfg),
                            demoter=HALODemoter(cfg, storage=st),
                            refetcher=HALORefetcher(cfg, storage=st), chunk_size=chunk,
                            recent_window=recent)


# ---------------------------------------------------------- chunk-walk identity
@pytest.mark.parametrize("T", [1, 16, 128, 1024])
@pytest.mark.parametrize("chunk", [1, 16, 64, 256, 1024])
def test_chunked_matches_reference(T, chunk):
    from halo_b200 import HALOCacheChunked as C
    q, k, v = _make_qkv(T=T)
    ref = _ref_attention(q, k, v)
    ro = rl = None
    for c0 in range(0, T, chunk):
        o, l = C._chunk_attention(q, k[..., c0:c0 + chunk, :], v[..., c0:c0 + chunk, :])
        ro, rl = (o, l) if ro is None else C._lse_merge(ro, rl, o, l)
    assert torch.allclose(ro.to(q.dtype), ref, atol=1e-5, rtol=1e-5)


def test_chunked_matches_reference_bf16():
    from halo_b200 import HALOCacheChunked as C
    q, k, v = _make_qkv(T=512, dtype=torch.bfloat16)
    ref = _ref_attention(q, k, v).to(torch.bfloat16)
    ro = rl = None
    for c0 in range(0, 512, 64):
        o, l = C._chunk_attention(q, k[..., c0:c0 + 64, :], v[..., c0:c0 + 64, :])
        ro, rl = (o, l) if ro is None else C._lse_merge(ro, rl, o, l)
    assert torch.allclose(ro.to(torch.bfloat16), ref, atol=5e-3, rtol=5e-3)


@pytest.mark.parametrize("H,H_kv", [(8, 1), (8, 2), (8, 4), (8, 8), (16, 2)])
def test_gqa_broadcasting(H, H_kv):
    from halo_b200 import HALOCacheChunked as C
    q, k, v = _make_qkv(H=H, H_kv=H_kv, T=64)
    out, _ = C._chunk_attention(q, k, v)
    assert torch.allclose(out, _ref_attention(q, k, v), atol=1e-5)


def test_chunk_attention_causal_mask_and_lse():
    """The static helper with the additive causal mask compute_attention
    builds, against the oracle (out and LSE)."""
    from halo_b200 import HALOCacheChunked as C
    g = torch.Generator().manual_seed(3)
    q = torch.randn(1, 4, 24, 32, generator=g)
    k = torch.randn(1, 2, 40, 32, generator=g)
    v = torch.randn(1, 2, 40, 32, generator=g)
    i = torch.arange(24).unsqueeze(-1)
    j = torch.arange(40).unsqueeze(0)
    allowed = j <= 10 + i
    mask = torch.where(allowed, 0.0, float("-inf"))
    out, lse = C._chunk_attention(q.to(DEV), k.to(DEV), v.to(DEV), causal_mask=mask.to(DEV))
    ro, rl = OA.chunk_attention(q, k, v, mask=allowed.view(1, 1, 24, 40))
    assert (out.cpu() - ro).abs().max() < 1e-5 and (lse.cpu() - rl).abs().max() < 1e-5


# ---------------------------------------------------------- cache plumbing
def test_identity_at_full_hot_ratio():
    cache = _cache(H_kv=2, D=32, chunk=64)
    q, k, v = _make_qkv(B=1, H=4, H_kv=2, T=200, D=32)
    cache.update(k, v, layer_idx=0)
    cache._mode = "chunked"
    q1 = q[..., :1, :]
    out = cache.compute_attention(q1, layer_idx=0)
    assert torch.allclose(out, _ref_attention(q1, k, v), atol=1e-5)


def test_telemetry_reports_chunk_count():
    cache = _cache(H_kv=4, D=32, chunk=128, hot_ratio=0.1)
    q, k, v = _make_qkv(T=1000)
    cache.update(k, v, layer_idx=0)
    cache._mode = "chunked"
    cache.compute_attention(q[..., -1:, :], layer_idx=0)
    tele = cache.telemetry()
    assert tele["chunked_n_layers_called"] == 1
    assert tele["chunked_used_lse_merge_any"] is True
    assert tele["chunked_total_chunks"] == (1000 + 127) // 128


@pytest.mark.parametrize("name", list(I.DECODE_CASES))
def test_compute_attention_cold_tier_matches_golden(name):
    """Cold rows installed in the pinned host tier, recent rows on the GPU;
    compute_attention streams the cold tier and must match the reference."""
    (q, k, v), T_cold, chunk = I.decode_inputs(name)
    g = I.load("attention.npz")[name]
    cache = _cache(H_kv=k.shape[1], D=k.shape[-1], chunk=chunk, dtype=k.dtype)
    cache.update(k[..., T_cold:, :].to(DEV), v[..., T_cold:, :].to(DEV), layer_idx=0)
    cache._mode = "chunked"
    cache._cold_k[0] = k[..., :T_cold, :]
    cache._cold_v[0] = v[..., :T_cold, :]
    cache.staging_slot_bytes = 64 * 1024          # force several staging slots
    out = cache.compute_attention(q.to(DEV), layer_idx=0)
    assert out.dtype == q.dtype
    tol = 1e-5 if q.dtype == torch.float32 else 1e-2   # out is rounded to q.dtype
    assert (out.float().cpu() - torch.from_numpy(g["out_qdtype"])).abs().max().item() <= tol
    assert cache.telemetry()["chunked_total_chunks"] == int(g["n_chunks"])
    assert cache.get_seq_length(0) == k.shape[-2]
    assert torch.equal(cache._cold_k[0], k[..., :T_cold, :])


@pytest.mark.parametrize("name", list(I.PREFILL_CASES))
def test_compute_attention_prefill_causal_matches_golden(name):
    (q, k, v), T_cold, chunk = I.prefill_inputs(name)
    g = I.load("attention.npz")[name]
    cache = _cache(H_kv=k.shape[1], D=k.shape[-1], chunk=chunk, dtype=k.dtype)
    cache.update(k[..., T_cold:, :].to(DEV), v[..., T_cold:, :].to(DEV), layer_idx=0)
    cache._mode = "chunked"
    cache._cold_k[0] = k[..., :T_cold, :]
    cache._cold_v[0] = v[..., :T_cold, :]
    out = cache.compute_attention(q.to(DEV), layer_idx=0)
    ref = torch.from_numpy(g["out"])
    tol = 1e-5 if q.dtype == torch.float32 else 1e-2
    assert (out.float().cpu() - ref).abs().max().item() <= tol


def test_peel_roundtrip_and_bounded_residency():
    """Decode-style updates: GPU rows stay <= recent_window + chunk_size,
    the peeled rows land bit-exact in the cold tier, attention stays exact."""
    torch.manual_seed(0)
    cache = _cache(H_kv=2, D=64, chunk=32, recent=8, dtype=torch.bfloat16)
    B, H, D = 2, 8, 64
    ks, vs = [], []
    k0 = torch.randn(B, 2, 100, D, device=DEV).bfloat16()
    v0 = torch.randn(B, 2, 100, D, device=DEV).bfloat16()
    cache.update(k0, v0, layer_idx=0)
    ks.append(k0); vs.append(v0)
    for step in range(60):
        kn = torch.randn(B, 2, 1, D, device=DEV).bfloat16()
        vn = torch.randn(B, 2, 1, D, device=DEV).bfloat16()
        K, _ = cache.update(kn, vn, layer_idx=0)
        ks.append(kn); vs.append(vn)
        assert cache._mode == "chunked"
        assert K.shape[-2] <= cache.recent_window + cache.chunk_size
    k_all, v_all = torch.cat(ks, -2), torch.cat(vs, -2)
    T_cold = cache._cold_k[0].shape[-2]
    assert torch.equal(cache._cold_k[0], k_all[..., :T_cold, :].cpu())
    assert torch.equal(cache._cold_v[0], v_all[..., :T_cold, :].cpu())
    assert cache.get_seq_length(0) == k_all.shape[-2]
    q = torch.randn(B, H, 1, D, device=DEV).bfloat16()
    out = cache.compute_attention(q, layer_idx=0)
    ref, _ = OA.full_attention_f64(q.cpu(), k_all.cpu(), v_all.cpu())
    assert (out.float().cpu() - ref.float()).abs().max().item() <= 1e-2


# ---------------------------------------------------------- triton_chunked names
def _ref_full(q, k, v, q_pos):
    o, _ = OA.full_attention_f64(q.cpu(), k.cpu(), v.cpu(), q_pos=q_pos.cpu())
    return o.float()


def _split(k, v, chunk, T):
    return [(k[..., c0:min(c0 + chunk, T), :].contiguous(), v[..., c0:min(c0 + chunk, T), :].contiguous(),
             c0, True) for c0 in range(0, T, chunk)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("chunk_size", [128, 512])
def test_triton_names_match_reference_small(dtype, chunk_size):
    from halo_b200.triton_chunked import triton_chunked_attention
    torch.manual_seed(0)
    B, H, H_kv, D, T = 1, 8, 2, 64, 1024
    q = (torch.randn(B, H, 1, D, device=DEV) * 0.1).to(dtype)
    k = (torch.randn(B, H_kv, T, D, device=DEV) * 0.1).to(dtype)
    v = (torch.randn(B, H_kv, T, D, device=DEV) * 0.1).to(dtype)
    q_pos = torch.tensor([T - 1], device=DEV)
    ref = _ref_full(q, k, v, q_pos)
    out = triton_chunked_attention(q, _split(k, v, chunk_size, T), scale=1 / math.sqrt(D), q_pos=q_pos)
    rel = ((ref - out.float().cpu()).norm() / ref.norm()).item()
    assert rel <= (1e-4 if dtype == torch.float32 else 5e-3)


def test_triton_names_single_launch_and_streamed():
    from halo_b200.triton_chunked import (triton_chunked_attention_single_launch,
                                          triton_chunked_attention_streamed, init_acc,
                                          update_chunk, finalize)
    torch.manual_seed(3)
    B, H, H_kv, D, T_cold, T_hot = 1, 8, 2, 64, 1024, 256
    T = T_cold + T_hot
    q = torch.randn(B, H, 1, D, device=DEV) * 0.1
    k = torch.randn(B, H_kv, T, D, device=DEV) * 0.1
    v = torch.randn(B, H_kv, T, D, device=DEV) * 0.1
    q_pos = torch.tensor([T - 1], device=DEV)
    ref = _ref_full(q, k, v, q_pos)
    rel = lambda o: ((ref - o.float().cpu()).norm() / ref.norm()).item()
    ck, cv = k[..., :T_cold, :].cpu().pin_memory(), v[..., :T_cold, :].cpu().pin_memory()
    hk, hv = k[..., T_cold:, :].contiguous(), v[..., T_cold:, :].contiguous()
    sc = 1 / math.sqrt(D)
    assert rel(triton_chunked_attention_single_launch(q, ck, cv, hk, hv, scale=sc, q_pos=q_pos)) <= 1e-4
    assert rel(triton_chunked_attention_single_launch(
        q, k.cpu().pin_memory(), v.cpu().pin_memory(), None, None, scale=sc, q_pos=q_pos)) <= 1e-4
    assert rel(triton_chunked_attention_single_launch(q, None, None, k.contiguous(), v.contiguous(),
                                                      scale=sc, q_pos=q_pos)) <= 1e-4
    cold = [(ck[..., c0:c0 + 256, :], cv[..., c0:c0 + 256, :], c0) for c0 in range(0, T_cold, 256)]
    hot = [(hk, hv, T_cold)]
    assert rel(triton_chunked_attention_streamed(q, cold, hot, scale=sc, q_pos=q_pos)) <= 1e-4
    m, l, o = init_acc(B=B, H=H, D_v=D, device=DEV)
    for kc, vc, c0, _ in _split(k, v, 300, T):
        update_chunk(q=q.squeeze(2), k=kc, v=vc, m=m, l=l, o=o, scale=sc, chunk_start=c0,
                     q_pos=q_pos, apply_causal=True)
    assert rel(finalize(m=m, l=l, o=o, out_dtype=q.dtype).unsqueeze(2)) <= 1e-4


def test_triton_names_noncontiguous_partition_and_permutation():
    from halo_b200.triton_chunked import triton_chunked_attention
    torch.manual_seed(4)
    B, H, H_kv, D, T = 1, 8, 2, 64, 2048
    q = torch.randn(B, H, 1, D, device=DEV) * 0.1
    k = torch.randn(B, H_kv, T, D, device=DEV) * 0.1
    v = torch.randn(B, H_kv, T, D, device=DEV) * 0.1
    q_pos = torch.tensor([T - 1], device=DEV)
    iv = [(0, 256), (768, 1024), (1280, 1408), (1536, 1664), (1856, 2048)]
    keep = torch.zeros(T, dtype=torch.bool)
    for a, b in iv:
        keep[a:b] = True
    ref, _ = OA.full_attention_f64(q.cpu(), k.cpu(), v.cpu(), q_pos=T - 1, keep=keep)
    ch = [(k[..., a:b, :].contiguous(), v[..., a:b, :].contiguous(), a, True) for a, b in iv]
    out = triton_chunked_attention(q, ch, scale=1 / math.sqrt(D), q_pos=q_pos)
    assert ((ref.float() - out.float().cpu()).norm() / ref.norm()).item() <= 1e-4
    random.seed(0)
    random.shuffle(ch)
    out2 = triton_chunked_attention(q, ch, scale=1 / math.sqrt(D), q_pos=q_pos)
    assert ((ref.float() - out2.float().cpu()).norm() / ref.norm()).item() <= 1e-4


# ---------------------------------------------------------- HF integration
def _tiny_qwen(attn="sdpa", vocab=256, seed=0):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    torch.manual_seed(seed)
    cfg = Qwen2Config(vocab_size=vocab, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=4096,
                      rope_theta=10000.0, tie_word_embeddings=False, attn_implementation=attn)
    return Qwen2ForCausalLM(cfg).eval().to(DEV)


def test_wrap_with_chunked_runs_generate_and_transitions():
    from halo_b200 import HALOConfig, HALOCacheChunked, wrap_with_halo
    model = _tiny_qwen()
    wrap_with_halo(model, HALOConfig(hot_ratio=0.5, chunked=True, chunk_size=32, recent_window=16,
                                     tiers=("dram",)))
    cache = model._halo_cache
    assert isinstance(cache, HALOCacheChunked) and cache._mode == "warmup"
    ids = torch.randint(0, 256, (1, 80), device=DEV)
    with torch.no_grad():
        out = model.generate(ids, max_new_tokens=5, do_sample=False)
    assert out.shape == (1, 85)
    assert cache._mode == "chunked"
    tele = cache.telemetry()
    assert tele.get("chunked_n_layers_called", 0) > 0 and tele.get("chunked_used_lse_merge_any")


@pytest.mark.parametrize("hot_ratio", [0.5, 0.25])
def test_path_d_identity_vs_full_attention(hot_ratio):
    """Reference tests/test_path_d_identity_chunked.py:70-110: Path D logits
    within 5e-4 of full attention in fp32 on a tiny Qwen2."""
    from halo_b200 import HALOConfig, wrap_with_halo
    model = _tiny_qwen(attn="eager", vocab=512).float()
    torch.manual_seed(1)
    prompt = torch.randint(10, 502, (1, 256), device=DEV)
    with torch.no_grad():
        ref = model(prompt, use_cache=False).logits[:, -1, :].clone()
    wrap_with_halo(model, HALOConfig(hot_ratio=hot_ratio, chunked=True, chunk_size=32, recent_window=8))
    cache = model._halo_cache
    with torch.no_grad():
        model(prompt[:, :-1], past_key_values=cache, use_cache=True)
        out = model(prompt[:, -1:], past_key_values=cache, use_cache=True).logits[:, -1, :]
    assert cache._mode == "chunked" and cache._cold_k
    assert (ref - out).abs().max().item() < 5e-4


def test_chunked_prefill_then_generate_matches_plain_decode():
    from halo_b200 import HALOConfig, wrap_with_halo
    from halo_b200.chunked_prefill import prefill_then_generate
    model = _tiny_qwen(attn="eager", vocab=512).float()
    torch.manual_seed(2)
    prompt = torch.randint(10, 502, (1, 300), device=DEV)
    with torch.no_grad():
        ref = model(prompt, use_cache=False).logits[:, -1, :]
    wrap_with_halo(model, HALOConfig(chunked=True, chunk_size=32, recent_window=8))
    res = prefill_then_generate(model, prompt, prefill_chunk_tokens=64, max_new_tokens=3)
    assert res["generated_ids"].shape == (1, 303)
    assert (res["step_logits"][0] - ref).abs().max().item() < 5e-4
    assert res["cache_telemetry"]["cold_layers"] == 2
