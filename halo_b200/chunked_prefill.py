"""Chunked prefill then decode (``halo/chunked_prefill.py`` in lzbaclz/HALO,
:49-205): the prompt goes through the model in slices with the cache forced
into chunked mode, every layer is peeled back to ``recent_window`` rows
between slices (bounded HBM residency), then a manual greedy / sampling
decode loop runs on the populated cache.  Each slice's attention is
``HALOCacheChunked.compute_attention`` with ``T_q > 1`` and causal masks.
"""
from __future__ import annotations

from typing import Optional


def _force_chunked_mode(cache) -> None:
    cache._mode = "chunked"


def _peel_all_layers(cache) -> None:
    todo = [i for i, _, k, _ in cache._iter_layer_kv()
            if k is not None and k.numel() > 0 and k.shape[-2] > cache.recent_window]
    for i in todo:
        cache._peel_to_cold(i)


def prefill_then_generate(model, input_ids, *, prefill_chunk_tokens: int = 1024,
                          max_new_tokens: int = 32, do_sample: bool = False,
                          temperature: float = 1.0, top_p: float = 1.0,
                          attention_mask=None) -> dict:
    """Prefill ``input_ids (1, T)`` in slices, then decode ``max_new_tokens``.
    Returns ``generated_ids``, peak-GPU figures, cache telemetry and the
    per-step logits, as the reference does."""
    import torch
    cache = model._halo_cache
    cache.reset()
    _force_chunked_mode(cache)
    dev = input_ids.device
    B, T = input_ids.shape
    assert B == 1, "chunked-prefill harness assumes batch=1"
    cuda = dev.type == "cuda"
    if cuda:
        torch.cuda.reset_peak_memory_stats()
    last_logits = None
    for pos in range(0, T, prefill_chunk_tokens):
        end = min(pos + prefill_chunk_tokens, T)
        with torch.no_grad():
            res = model(input_ids=input_ids[:, pos:end], past_key_values=cache,
                        cache_position=torch.arange(pos, end, device=dev), use_cache=True,
                        return_dict=True)
        if end == T:
            last_logits = res.logits[:, -1, :].detach().clone()
        del res
        _peel_all_layers(cache)
    prefill_peak = torch.cuda.max_memory_allocated() / 2 ** 30 if cuda else 0.0
    if cuda:
        torch.cuda.reset_peak_memory_stats()

    def pick(lg):
        if not do_sample:
            return lg.argmax(dim=-1, keepdim=True)
        probs = torch.softmax(lg / max(temperature, 1e-6), dim=-1)
        if top_p < 1.0:
            sp, si = probs.sort(dim=-1, descending=True)
            drop = sp.cumsum(dim=-1) > top_p
            drop[..., 0] = False
            sp = sp.masked_fill(drop, 0.0)
            sp = sp / sp.sum(dim=-1, keepdim=True)
            return si.gather(-1, torch.multinomial(sp, 1))
        return torch.multinomial(probs, 1)

    generated, step_logits, logits = [], [], last_logits
    for _ in range(max_new_tokens):
        step_logits.append(logits.detach().clone())
        tok = pick(logits)
        generated.append(tok)
        with torch.no_grad():
            res = model(input_ids=tok, past_key_values=cache,
                        cache_position=torch.tensor([cache.get_seq_length()], device=dev),
                        use_cache=True, return_dict=True)
        logits = res.logits[:, -1, :]
        del res
        _peel_all_layers(cache)
    decode_peak = torch.cuda.max_memory_allocated() / 2 ** 30 if cuda else 0.0
    return {"generated_ids": torch.cat([input_ids] + generated, dim=-1),
            "prefill_peak_gib": prefill_peak, "decode_peak_gib": decode_peak,
            "overall_peak_gib": max(prefill_peak, decode_peak),
            "cache_telemetry": cache.telemetry(), "step_logits": step_logits}


__all__ = ["prefill_then_generate"]
