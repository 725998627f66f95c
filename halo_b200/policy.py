"""Public configuration and wiring: ``HALOConfig`` and ``wrap_with_halo``.

Mirrors ``halo/policy.py`` of lzbaclz/HALO (:37-478): the same dataclass
fields and defaults, ``HALO_OVERRIDES`` parsing, the ``halo_chunked``
attention interface registered in transformers' ``ALL_ATTENTION_FUNCTIONS``
and the ``generate`` hook that threads the cache through.  The chunked
(Path D) cache is ``halo_b200.kv_cache_chunked.HALOCacheChunked``; the
eviction variant (Path C) is not part of this package.
"""
from __future__ import annotations

import ast
import math
import os
from dataclasses import dataclass, field, replace
from typing import Any, Optional, Sequence

from halo_b200.demoter import HALODemoter
from halo_b200.kv_cache import HALOCache
from halo_b200.memory_tier import MemoryTier, TieredStorage
from halo_b200.refetcher import HALORefetcher
from halo_b200.scorer import HALOScorer


@dataclass
class HALOConfig:
    """User-facing configuration (fields and defaults as in the reference,
    ``halo/policy.py:46-126``)."""

    hot_ratio: float = 0.10
    score_alpha: float = 1.0
    score_beta: float = 0.5
    score_gamma: float = 2.0
    sink_tokens: int = 4
    refresh_window: int = 64
    tiers: Sequence[str] = ("gpu", "dram")
    block_size: int = 32
    nvme_path: Optional[str] = None
    async_refetch: bool = True
    lookahead: int = 1
    layerwise_budget: str = "uniform"
    eviction: bool = False
    chunked: bool = False
    chunk_size: int = 512
    recent_window: int = 64
    use_triton: bool = False
    log_dir: Optional[str] = None
    extra: dict = field(default_factory=dict)

    def make_storage(self, *, num_layers: int, num_kv_heads: int, head_dim: int, dtype, device):
        return TieredStorage(tiers=[MemoryTier.from_name(t) for t in self.tiers],
                             num_layers=num_layers, num_kv_heads=num_kv_heads, head_dim=head_dim,
                             block_size=self.block_size, dtype=dtype, device=device,
                             nvme_path=self.nvme_path)

    def with_overrides(self, overrides: dict) -> "HALOConfig":
        """Copy with known fields replaced; unknown keys land in ``extra``."""
        known = set(self.__dataclass_fields__)
        upd = {k: v for k, v in overrides.items() if k in known}
        unknown = {k: v for k, v in overrides.items() if k not in known}
        if unknown:
            upd["extra"] = {**self.extra, **unknown}
        return replace(self, **upd)


def parse_overrides(s: Optional[str] = None) -> dict[str, Any]:
    """Parse ``"k1=v1,k2=[a,b],k3='x,y'"`` (default: ``$HALO_OVERRIDES``).

    Top-level commas split pairs; commas inside brackets or quotes do not.
    Values go through ``ast.literal_eval`` and stay strings when that fails
    (``halo/policy.py:163-212``)."""
    if s is None:
        s = os.environ.get("HALO_OVERRIDES", "")
    s = s.strip()
    if not s:
        return {}
    parts, cur, depth, quote = [], [], 0, None
    for ch in s:
        if quote:
            cur.append(ch)
            if ch == quote and (len(cur) < 2 or cur[-2] != "\\"):
                quote = None
            continue
        if ch in "'\"":
            quote = ch
        elif ch in "([{":
            depth += 1
        elif ch in ")]}":
            depth -= 1
        elif ch == "," and depth == 0:
            parts.append("".join(cur).strip())
            cur = []
            continue
        cur.append(ch)
    if cur:
        parts.append("".join(cur).strip())
    out: dict = {}
    for kv in parts:
        if "=" not in kv:
            continue
        k, v = (x.strip() for x in kv.split("=", 1))
        try:
            out[k] = ast.literal_eval(v)
        except (ValueError, SyntaxError):
            out[k] = v
    return out


def wrap_with_halo(model, config: Optional[HALOConfig] = None):
    """Install HALO's cache on a HuggingFace causal LM (in place).

    With ``config.chunked`` the cache is :class:`HALOCacheChunked` and the
    model's attention goes through the ``halo_chunked`` interface, i.e. the
    B200 split-KV kernels.  Raises ``ValueError`` when ``model.config`` is
    missing or when ``chunked`` and ``eviction`` are both set
    (``halo/policy.py:220-313``)."""
    config = config or HALOConfig()
    env = parse_overrides()
    if env:
        config = config.with_overrides(env)
    cfg = getattr(model, "config", None)
    if cfg is None:
        raise ValueError("`model.config` is missing; cannot wire HALO without architecture metadata.")
    num_layers = getattr(cfg, "num_hidden_layers", None) or getattr(cfg, "n_layer")
    num_kv_heads = getattr(cfg, "num_key_value_heads", None) or getattr(cfg, "num_attention_heads")
    head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    p0 = next(model.parameters())
    if config.chunked and config.eviction:
        raise ValueError("HALOConfig: `chunked` (Path D) and `eviction` (Path C) are mutually exclusive.")
    if config.eviction:
        raise ValueError("HALOConfig(eviction=True) (Path C) is not part of halo_b200.")
    storage = config.make_storage(num_layers=num_layers, num_kv_heads=num_kv_heads,
                                  head_dim=head_dim, dtype=p0.dtype, device=p0.device)
    scorer = HALOScorer(config)
    demoter = HALODemoter(config, storage=storage)
    refetcher = HALORefetcher(config, storage=storage)
    if config.chunked:
        from halo_b200.kv_cache_chunked import HALOCacheChunked
        cache = HALOCacheChunked(config=config, storage=storage, scorer=scorer, demoter=demoter,
                                 refetcher=refetcher, chunk_size=config.chunk_size,
                                 recent_window=config.recent_window, use_triton=config.use_triton)
    else:
        cache = HALOCache(config=config, storage=storage, scorer=scorer, demoter=demoter,
                          refetcher=refetcher)
    model._halo_config = config
    model._halo_cache = cache
    model._halo_scorer = scorer
    model._halo_demoter = demoter
    model._halo_refetcher = refetcher
    model._halo_storage = storage
    _install_generate_hook(model)
    if config.chunked:
        _install_chunked_attention_interface(model, cache)
    return model


def _install_chunked_attention_interface(model, cache) -> None:
    """Register ``ALL_ATTENTION_FUNCTIONS["halo_chunked"]`` bound to ``cache``
    and switch the model (and every submodule config) to it
    (``halo/policy.py:321-395``).  Warm-up mode delegates to transformers'
    ``sdpa``; chunked mode calls ``cache.compute_attention``."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    def halo_chunked_interface(module, query, key, value, attention_mask=None, dropout=0.0,
                               scaling=None, **kwargs):
        if cache._mode == "warmup":
            out = cache._one_shot_attention_for_module(module, query, key, value,
                                                       attention_mask=attention_mask,
                                                       scaling=scaling)
            return out, None
        out = cache.compute_attention(query, layer_idx=module.layer_idx, scaling=scaling)
        return out.transpose(1, 2).contiguous(), None

    ALL_ATTENTION_FUNCTIONS["halo_chunked"] = halo_chunked_interface
    model.config._attn_implementation = "halo_chunked"
    for mod in model.modules():
        if mod is not model and hasattr(mod, "config"):
            try:
                mod.config._attn_implementation = "halo_chunked"
            except Exception:
                pass
    _attach_one_shot_fallback(cache)


def _attach_one_shot_fallback(cache) -> None:
    """Give the cache a warm-up attention: transformers' registered ``sdpa``
    (byte-identical to the unwrapped model), else plain SDPA."""
    import types

    def one_shot(self_, module, query, key, value, *, attention_mask=None, scaling=None, **kw):
        try:
            from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
            out, _ = ALL_ATTENTION_FUNCTIONS["sdpa"](module, query, key, value, attention_mask,
                                                      dropout=0.0, scaling=scaling, **kw)
            return out
        except Exception:
            import torch
            H, H_kv = query.shape[1], key.shape[1]
            if H != H_kv:
                key = key.repeat_interleave(H // H_kv, dim=1)
                value = value.repeat_interleave(H // H_kv, dim=1)
            scaling = scaling if scaling is not None else 1.0 / math.sqrt(query.shape[-1])
            out = torch.nn.functional.scaled_dot_product_attention(
                query, key, value, attn_mask=attention_mask, dropout_p=0.0,
                is_causal=attention_mask is None and query.shape[-2] > 1, scale=scaling)
            return out.transpose(1, 2).contiguous()

    cache._one_shot_attention_for_module = types.MethodType(one_shot, cache)


def _install_generate_hook(model) -> None:
    """Wrap ``model.generate`` to inject (and reset) the HALO cache unless the
    caller passes that same cache (``halo/policy.py:450-478``)."""
    if getattr(model, "_halo_generate_patched", False):
        return
    original = model.generate

    def halo_generate(*args, **kwargs):
        cache = model._halo_cache
        if kwargs.get("past_key_values") is not cache:
            cache.reset()
            kwargs.setdefault("past_key_values", cache)
        kwargs.setdefault("use_cache", True)
        return original(*args, **kwargs)

    model.generate = halo_generate
    model._halo_generate_patched = True


__all__ = ["HALOConfig", "parse_overrides", "wrap_with_halo"]
