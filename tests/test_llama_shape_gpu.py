"""The drop-in path on a random-weight Llama-3-8B-shaped model (hidden 4096,
32 q-heads / 8 KV heads, head_dim 128, MLP 14336, vocabulary 128256, bf16;
two decoder layers, no checkpoint): ``wrap_with_halo(HALOConfig(chunked=
True))`` and ``prefill_then_generate`` over a 16384-token prompt in slices of
4096 (``halo/chunked_prefill.py:73-205``, ``halo/policy.py:220-373``;
the reference tests ``tests/test_chunked_wrap_integration.py:55-134`` and
``tests/test_path_d_identity_chunked.py:70-138`` do the same on a tiny
Qwen2).  Each slice's attention runs the tensor-core prefill kernel over
the cold tier (staged from pinned host memory) and the recent rows, then
decode steps run the split-KV kernel.

Checker: the same weights with torch's SDPA over the whole sequence.  The
last-position logits of the prompt and of the first decode step are
compared in float32 (SDPA run in fp32 on an fp32 copy of the weights) for
both the HALO path and SDPA in bf16: HALO's error must stay within that of
bf16 SDPA itself (plus a small margin) and pick the same top token."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
T_PROMPT, SLICE = 16384, 4096


def _model():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336,
                      num_hidden_layers=2, num_attention_heads=32, num_key_value_heads=8,
                      head_dim=128, max_position_embeddings=T_PROMPT + 64, rope_theta=500000.0,
                      tie_word_embeddings=False, attn_implementation="sdpa")
    torch.manual_seed(0)
    with torch.device(DEV):
        model = LlamaForCausalLM(cfg)
    return model.to(torch.bfloat16).eval()


def _last_logits(model, ids):
    with torch.no_grad():
        return model(ids, use_cache=False, logits_to_keep=1).logits[:, -1, :].float()


def _rel(a, b):
    return ((a - b).norm() / b.norm()).item()


def test_llama_shaped_chunked_prefill_and_decode_match_full_attention():
    from halo_b200 import HALOConfig, _lib as L, wrap_with_halo
    from halo_b200.chunked_prefill import prefill_then_generate
    model = _model()
    g = torch.Generator(device=DEV).manual_seed(1)
    ids = torch.randint(0, 128256, (1, T_PROMPT), device=DEV, generator=g)

    # references: SDPA in bf16 and in fp32 over the whole prompt, and over
    # the prompt + the token the HALO run picks next
    ref16 = _last_logits(model, ids)
    model.float()
    ref32 = _last_logits(model, ids)
    model.to(torch.bfloat16)
    torch.cuda.empty_cache()

    cfg = HALOConfig(chunked=True, chunk_size=1024, recent_window=64, tiers=("gpu", "dram"))
    wrap_with_halo(model, cfg)
    cache = model._halo_cache
    n0 = L.launch_count()
    res = prefill_then_generate(model, ids, prefill_chunk_tokens=SLICE, max_new_tokens=2)
    launches = L.launch_count() - n0
    halo0, halo1 = res["step_logits"][0].float(), res["step_logits"][1].float()
    tok = res["generated_ids"][:, T_PROMPT:T_PROMPT + 1]

    # residency stays bounded: after every slice and step the GPU holds at
    # most recent_window + one slice of rows per layer; the rest is cold
    tele = res["cache_telemetry"]
    assert tele["mode"] == "chunked" and tele["cold_layers"] == 2
    for _i, _layer, k, _v in cache._iter_layer_kv():
        assert k is None or k.shape[-2] <= cfg.recent_window + 1
    assert tele["cold_positions_per_layer_max"] >= T_PROMPT + 1 - cfg.recent_window - 1
    # each slice of each layer ran the prefill kernel (fp16 V copy + kp3),
    # and decode ran the split-KV kernels
    assert launches >= 2 * (T_PROMPT // SLICE) * 2

    # prompt logits: HALO within bf16 SDPA's own error (vs fp32 SDPA)
    e_sdpa, e_halo = _rel(ref16, ref32), _rel(halo0, ref32)
    assert e_halo <= max(2.0 * e_sdpa, 5e-3), (e_halo, e_sdpa)
    assert halo0.argmax().item() == ref32.argmax().item()

    # first decode step (cold tier + recent rows, split-KV decode)
    ids1 = torch.cat([ids, tok], dim=1)
    cfg_attn = model.config._attn_implementation
    model.config._attn_implementation = "sdpa"
    try:
        r16 = _last_logits(model, ids1)
        model.float()
        r32 = _last_logits(model, ids1)
        model.to(torch.bfloat16)
    finally:
        model.config._attn_implementation = cfg_attn
    e_sdpa1, e_halo1 = _rel(r16, r32), _rel(halo1, r32)
    assert e_halo1 <= max(2.0 * e_sdpa1, 5e-3), (e_halo1, e_sdpa1)
    assert halo1.argmax().item() == r32.argmax().item()
    assert L.device_error() == 0
