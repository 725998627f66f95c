"""Host-side configuration and wiring (no GPU): ``HALOConfig`` defaults,
``parse_overrides`` and ``with_overrides`` against the reference's own
results (``tests/golden/policy.json``, made by ``make_golden.py`` from
halo/policy.py:37-212), the ``ValueError`` rules of ``wrap_with_halo``
(:248-286), and that the chunked cache refuses CPU tensors instead of
computing attention on the host."""
from __future__ import annotations

import dataclasses
import json
import os

import pytest
import torch

import inputs as I
from halo_b200.policy import HALOConfig, parse_overrides, wrap_with_halo


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(I.HERE, "policy.json")) as f:
        return json.load(f)


def _fields(cfg: HALOConfig) -> dict:
    return {f.name: repr(getattr(cfg, f.name)) for f in dataclasses.fields(cfg)}


def test_config_fields_and_defaults_match_reference(golden):
    assert _fields(HALOConfig()) == golden["defaults"]


def test_parse_overrides_matches_reference(golden):
    assert len(golden["parse_overrides"]) == len(I.OVERRIDE_CASES)
    for s, want in zip(I.OVERRIDE_CASES, golden["parse_overrides"]):
        assert repr(parse_overrides(s)) == want, s


def test_with_overrides_matches_reference(golden):
    for d, want in zip(I.WITH_OVERRIDES_CASES, golden["with_overrides"]):
        assert _fields(HALOConfig().with_overrides(d)) == want, d


def test_parse_overrides_reads_environment(monkeypatch):
    monkeypatch.setenv("HALO_OVERRIDES", "  hot_ratio=0.3,tiers=['gpu']  ")
    assert parse_overrides() == {"hot_ratio": 0.3, "tiers": ["gpu"]}
    monkeypatch.delenv("HALO_OVERRIDES")
    assert parse_overrides() == {}


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=64, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=512)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).eval()


class _NoConfig(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.w = torch.nn.Linear(2, 2)


def test_wrap_without_model_config_raises():
    with pytest.raises(ValueError):
        wrap_with_halo(_NoConfig(), HALOConfig(chunked=True))


def test_wrap_chunked_and_eviction_raises():
    with pytest.raises(ValueError):
        wrap_with_halo(_tiny_llama(), HALOConfig(chunked=True, eviction=True))


def test_wrap_installs_cache_and_environment_overrides(monkeypatch):
    monkeypatch.setenv("HALO_OVERRIDES", "chunk_size=16,recent_window=8,my_knob=3")
    m = wrap_with_halo(_tiny_llama(), HALOConfig(chunked=True))
    assert m._halo_config.chunk_size == 16 and m._halo_config.recent_window == 8
    assert m._halo_config.extra == {"my_knob": 3}
    cache = m._halo_cache
    assert type(cache).__name__ == "HALOCacheChunked"
    assert cache._mode == "warmup" and cache.chunk_size == 16 and cache.recent_window == 8
    for attr in ("_halo_scorer", "_halo_demoter", "_halo_refetcher", "_halo_storage"):
        assert getattr(m, attr) is not None
    assert m.config._attn_implementation == "halo_chunked"


def test_chunked_cache_refuses_cpu_tensors():
    """No host fallback: once the context is long enough for chunked mode,
    the cache raises on CPU tensors rather than attending on the CPU."""
    m = wrap_with_halo(_tiny_llama(), HALOConfig(chunked=True, chunk_size=16, recent_window=8))
    ids = torch.randint(0, 64, (1, 40), generator=torch.Generator().manual_seed(1))
    with pytest.raises(RuntimeError, match="CUDA"):
        m.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=2, do_sample=False,
                   pad_token_id=0)


def test_unchunked_wrap_is_identity_at_full_hot_ratio():
    """Path A (``HALOCache``, no chunking) passes the ``DynamicCache`` rows
    through untouched: greedy decoding with the wrapped model equals the
    unwrapped one (the identity claim of the reference's
    ``tests/test_integration_identity.py``, on a random-weight model)."""
    base = _tiny_llama()
    ids = torch.randint(0, 64, (1, 24), generator=torch.Generator().manual_seed(3))
    mask = torch.ones_like(ids)
    with torch.no_grad():
        want = base.generate(ids, attention_mask=mask, max_new_tokens=8, do_sample=False,
                             pad_token_id=0)
    m = wrap_with_halo(_tiny_llama(), HALOConfig(hot_ratio=1.0))
    assert type(m._halo_cache).__name__ == "HALOCache"
    with torch.no_grad():
        got = m.generate(ids, attention_mask=mask, max_new_tokens=8, do_sample=False,
                         pad_token_id=0)
    assert torch.equal(got, want)
