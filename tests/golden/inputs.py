"""Seeded inputs shared by ``make_golden.py`` and the tests.

Golden fixtures store the reference's OUTPUTS and a SHA-256 digest of the
inputs; the inputs themselves are regenerated here from their seeds
(``torch.Generator`` on the CPU), so fixtures stay small.  A digest mismatch
means the generator changed and the fixtures must be regenerated.
"""
from __future__ import annotations

import hashlib
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# name: (B, H, H_kv, T, D, chunk, dtype, seed) -- T_q = 1 chunk walks
WALK_CASES = {
    "walk_f32_gqa4": (2, 8, 2, 300, 64, 64, torch.float32, 1),
    "walk_f32_mha": (1, 4, 4, 128, 32, 16, torch.float32, 2),
    "walk_f32_t1": (1, 4, 2, 1, 32, 16, torch.float32, 3),
    "walk_bf16_gqa4": (2, 16, 4, 520, 128, 128, torch.bfloat16, 4),
    "walk_bf16_gqa8": (1, 16, 2, 1000, 128, 256, torch.bfloat16, 5),
    "walk_f16_gqa4": (1, 8, 2, 256, 64, 64, torch.float16, 6),
}

# name: (B, H, H_kv, T_cold, T_gpu, D, chunk, dtype, seed) -- compute_attention T_q = 1
DECODE_CASES = {
    "decode_f32": (1, 8, 2, 700, 90, 32, 128, torch.float32, 21),
    "decode_bf16": (2, 8, 2, 1024, 64, 64, 256, torch.bfloat16, 22),
}

# name: (B, H, H_kv, T_cold, T_gpu, T_q, D, chunk, dtype, seed) -- T_q > 1 causal
PREFILL_CASES = {
    "prefill_f32": (1, 4, 2, 192, 80, 48, 32, 64, torch.float32, 11),
    "prefill_bf16": (1, 8, 2, 256, 128, 96, 64, 64, torch.bfloat16, 12),
}

# name: (shape, dtype, bits, seed)
KIVI_CASES = {
    "kivi_f16_b2": ((2, 3, 70, 128), torch.float16, 2, 31),
    "kivi_f16_b4": ((1, 2, 40, 64), torch.float16, 4, 32),
    "kivi_bf16_b2": ((1, 4, 50, 128), torch.bfloat16, 2, 33),
}

# name: (B, H, H_kv, T, D, page, dtype, seed, memory_ratio, min_pages)
SCORER_CASES = {
    "quest_f32_gqa4": (2, 8, 2, 130, 32, 16, torch.float32, 41, 4.0, 2),
    "quest_bf16_gqa4": (2, 16, 4, 512, 128, 32, torch.bfloat16, 42, 4.0, 4),
    "quest_bf16_gqa3": (1, 6, 2, 256, 64, 16, torch.bfloat16, 43, 2.0, 1),
}


def digest(*ts) -> str:
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def qkv(B, H, H_kv, T, D, dtype, seed, T_q=1):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, T_q, D, generator=g).to(dtype)
    k = torch.randn(B, H_kv, T, D, generator=g).to(dtype)
    v = torch.randn(B, H_kv, T, D, generator=g).to(dtype)
    return q, k, v


def walk_inputs(name):
    B, H, H_kv, T, D, chunk, dtype, seed = WALK_CASES[name]
    return qkv(B, H, H_kv, T, D, dtype, seed), chunk


def decode_inputs(name):
    B, H, H_kv, T_cold, T_gpu, D, chunk, dtype, seed = DECODE_CASES[name]
    return qkv(B, H, H_kv, T_cold + T_gpu, D, dtype, seed), T_cold, chunk


def prefill_inputs(name):
    B, H, H_kv, T_cold, T_gpu, T_q, D, chunk, dtype, seed = PREFILL_CASES[name]
    return qkv(B, H, H_kv, T_cold + T_gpu, D, dtype, seed, T_q=T_q), T_cold, chunk


def config1_inputs():
    """The fp32 CPU-runnable decode case: B1, H32/H_kv8, D128, T8192, seed 0."""
    g = torch.Generator().manual_seed(0)
    q = torch.randn(1, 32, 1, 128, generator=g)
    k = torch.randn(1, 8, 8192, 128, generator=g)
    v = torch.randn(1, 8, 8192, 128, generator=g)
    return q, k, v


def kivi_inputs(name):
    shape, dtype, bits, seed = KIVI_CASES[name]
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g)
    x[..., 3] *= 10.0                       # outlier channels
    x[..., 77 % shape[-1]] *= 10.0
    x[0, 0, 0, :32] = 0.5                   # constant group
    x[0, 0, 1, :32] = torch.linspace(0, 1e-3, 32)    # tiny range
    x[0, 0, 2, 32:64] = 6.0e4 * torch.sign(torch.randn(32, generator=g))  # huge range
    return x.to(dtype), bits


def scorer_inputs(name):
    B, H, H_kv, T, D, page, dtype, seed, mr, mp = SCORER_CASES[name]
    g = torch.Generator().manual_seed(seed)
    K = torch.randn(B, H_kv, T, D, generator=g)
    idx = torch.randperm(D, generator=g)[:4]
    K[..., idx] *= 10.0                     # 4 outlier channels x10
    K = K.to(dtype)
    q = torch.randn(B, H, 1, D, generator=g).to(dtype)
    return K, q, page, mr, mp


# HALOPress ablation scorer (baselines/scorer_ablations.py:184-268):
# name -> (B, H, H_kv, T, D, page, dtype, seed, memory_ratio, min_pages,
#          alpha, beta, gamma, sink_tokens, refresh_window)
PRESS_CASES = {
    "press_f32_gqa4": (2, 8, 2, 130, 32, 16, torch.float32, 51, 4.0, 2, 1.0, 0.5, 2.0, 4, 64),
    "press_bf16_gqa4": (2, 16, 4, 512, 128, 32, torch.bfloat16, 52, 4.0, 4, 1.0, 0.5, 2.0, 4, 8),
    "press_bf16_gqa3_tq2": (1, 6, 2, 256, 64, 16, torch.bfloat16, 53, 2.0, 1, 0.7, 1.5, 0.0, 40, 3),
}


def press_inputs(name):
    B, H, H_kv, T, D, page, dtype, seed, mr, mp, a, b, c, sink, win = PRESS_CASES[name]
    g = torch.Generator().manual_seed(seed)
    K = torch.randn(B, H_kv, T, D, generator=g)
    idx = torch.randperm(D, generator=g)[:4]
    K[..., idx] *= 10.0
    K = K.to(dtype)
    T_q = 2 if name.endswith("tq2") else 1
    q = torch.randn(B, H, T_q, D, generator=g).to(dtype)
    cfg = dict(page_size=page, memory_ratio=mr, min_pages_selected=mp, halopress_alpha=a,
               halopress_beta=b, halopress_gamma=c, halopress_sink_tokens=sink,
               halopress_refresh_window=win)
    return K, q, cfg


# ``HALO_OVERRIDES`` strings for ``parse_overrides`` (halo/policy.py:163-212):
# plain literals, strings that are not literals, nested brackets, quoted
# commas, escaped quotes, empty and key-less pairs, '=' inside a value.
OVERRIDE_CASES = [
    "",
    "   ",
    "hot_ratio=0.05",
    "tiers=[gpu, dram]",
    "tiers=['gpu','dram','nvme'],block_size=16",
    " chunked=True , chunk_size=1024 ,recent_window=128 ",
    "name='a,b',x=(1,2),y={'k': [1, 2]}",
    "bad, z=3",
    "path=/tmp/x=y",
    "q=\"it's\"",
    "a=1,,b=2",
    "esc='a\\',b',c=4",
    "nested=[[1,2],[3,(4,5)]],t=None,f=-1e-3",
    "unknown_knob=7,hot_ratio=0.5",
]

# ``HALOConfig().with_overrides(d)`` inputs (halo/policy.py:139-155): known
# fields are replaced, the rest lands in ``extra``.
WITH_OVERRIDES_CASES = [
    {},
    {"hot_ratio": 0.25, "chunked": True},
    {"tiers": ("gpu", "dram", "nvme"), "nvme_path": "/tmp/halo"},
    {"mystery": 1, "another": "x"},
    {"chunk_size": 2048, "mystery": [1, 2]},
]


# Host control flow (halo/scorer.py, refetcher.py, demoter.py, kv_cache.py,
# memory_tier.py): the configuration of the reference's unit-test fixtures,
# hotness snapshots (K, step, seed) and a multi-step update_hotness trace.
HOST_CONFIG = dict(hot_ratio=0.25, score_alpha=1.0, score_beta=0.5, score_gamma=2.0,
                   sink_tokens=2, refresh_window=8, tiers=("gpu", "dram"), block_size=4,
                   async_refetch=False, lookahead=1)
HOST_SCORE_CASES = [(64, 0, 0), (64, 10, 1), (37, 100, 2), (5, 3, 3), (1, 0, 4), (200, 7, 5)]
HOST_TRACE = dict(layers=2, K=64, steps=6, max_blocks=16, head_dim=8, kv_heads=2)


def host_attention(K: int, seed: int) -> torch.Tensor:
    """A head-mean attention snapshot: softmax of seeded N(0, 1) logits."""
    g = torch.Generator().manual_seed(seed)
    return torch.softmax(torch.randn(K, generator=g), dim=0)


def host_trace_attention(step: int, layer: int, K: int) -> torch.Tensor:
    """Trace snapshots: a window of extra mass sweeps the context (front to
    back, then wraps), so hot sets change and blocks move both ways."""
    base = host_attention(K, 1000 + 10 * step + layer)
    focus = torch.zeros(K)
    lo = (step * K // 4) % K
    focus[lo:lo + K // 4] = 1.0
    a = base + 4.0 * focus / focus.sum()
    return a / a.sum()


def load(name: str) -> dict:
    """Load ``tests/golden/<name>.npz`` as ``{case: {key: array}}``."""
    out: dict = {}
    with np.load(os.path.join(HERE, name), allow_pickle=False) as z:
        for full in z.files:
            case, key = full.split("/", 1)
            out.setdefault(case, {})[key] = z[full]
    return out
