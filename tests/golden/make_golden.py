"""Generate golden vectors by running the REFERENCE's own Python code.

Run in the build container, where a reference checkout is importable:

    python tests/golden/make_golden.py --reference <path-to-lzbaclz/HALO>

It imports ``halo.kv_cache_chunked.HALOCacheChunked`` (``_chunk_attention``,
``_lse_merge``, ``compute_attention``), ``baselines.kivi_cache``
(``_quantize_per_group`` / ``_dequantize_per_group``) and
``baselines.quest_path_d._QuestScorerAdapter``, the ablation scorers of
``baselines.scorer_ablations`` and ``halo.policy`` (``HALOConfig``,
``parse_overrides``) from the reference, runs them on the seeded inputs of
``tests/golden/inputs.py`` and stores their outputs plus an input digest in
``tests/golden/*.npz`` (the policy results, as ``repr`` strings, in
``tests/golden/policy.json``).  The GPU box has no reference
checkout; tests only read the committed fixtures.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
import warnings

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import inputs as I  # noqa: E402


def bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def ref_walk(C, q, chunks, scale=None):
    """The reference torch loop over ``(k, v, additive_mask)`` chunks:
    ``_chunk_attention`` then ``_lse_merge`` (kv_cache_chunked.py:900-908)."""
    ro = rl = None
    for k, v, mask in chunks:
        o, l = C._chunk_attention(q, k, v, scaling=scale, causal_mask=mask)
        if ro is None:
            ro, rl = o, l
        else:
            ro, rl = C._lse_merge(ro, rl, o, l)
    return ro, rl


def split(k, v, T0, T1, chunk):
    return [(k[..., c0:min(c0 + chunk, T1), :], v[..., c0:min(c0 + chunk, T1), :])
            for c0 in range(T0, T1, chunk)]


def gen_walk(C) -> dict:
    out = {}
    for name in I.WALK_CASES:
        (q, k, v), chunk = I.walk_inputs(name)
        o, l = ref_walk(C, q, [(kc, vc, None) for kc, vc in split(k, v, 0, k.shape[-2], chunk)])
        out[name] = {"digest": np.bytes_(I.digest(q, k, v)),
                     "out": o.numpy().astype(np.float32), "lse": l.numpy().astype(np.float32)}
    return out


def seed_cache(make_cache, q, k, v, T_cold, chunk):
    cache = make_cache(chunk, k.shape[1], k.shape[-1], k.dtype)
    cache.update(k[..., T_cold:, :], v[..., T_cold:, :], layer_idx=0)
    cache._mode = "chunked"
    cache._cold_k[0] = k[..., :T_cold, :].clone()
    cache._cold_v[0] = v[..., :T_cold, :].clone()
    return cache


def gen_decode(C, make_cache) -> dict:
    out = {}
    for name in I.DECODE_CASES:
        (q, k, v), T_cold, chunk = I.decode_inputs(name)
        T = k.shape[-2]
        cache = seed_cache(make_cache, q, k, v, T_cold, chunk)
        res = cache.compute_attention(q, layer_idx=0)
        n_chunks = cache.telemetry()["chunked_total_chunks"]
        chunks = split(k, v, 0, T_cold, chunk) + [
            (kc, vc) for kc, vc in split(k[..., T_cold:, :], v[..., T_cold:, :], 0, T - T_cold, chunk)]
        o, l = ref_walk(C, q, [(kc, vc, None) for kc, vc in chunks])
        out[name] = {"digest": np.bytes_(I.digest(q, k, v)), "n_chunks": np.int64(n_chunks),
                     "out_qdtype": res.float().numpy().astype(np.float32),
                     "out": o.numpy().astype(np.float32), "lse": l.numpy().astype(np.float32)}
    return out


def gen_prefill(C, make_cache) -> dict:
    """compute_attention with T_q > 1 (the chunked-prefill branch,
    kv_cache_chunked.py:873-942) through the reference cache plumbing."""
    out = {}
    for name in I.PREFILL_CASES:
        (q, k, v), T_cold, chunk = I.prefill_inputs(name)
        T, T_q = k.shape[-2], q.shape[-2]
        cache = seed_cache(make_cache, q, k, v, T_cold, chunk)
        res = cache.compute_attention(q, layer_idx=0)
        qpo = T - T_q
        chunks = []
        for base_k, base_v, Tp, off in ((k[..., :T_cold, :], v[..., :T_cold, :], T_cold, 0),
                                        (k[..., T_cold:, :], v[..., T_cold:, :], T - T_cold, T_cold)):
            for c0 in range(0, Tp, chunk):
                c1 = min(c0 + chunk, Tp)
                i = torch.arange(T_q).unsqueeze(-1)
                j = torch.arange(c1 - c0).unsqueeze(0)
                allowed = (off + c0 + j) <= (qpo + i)
                if not bool(allowed.any()):
                    continue
                mask = None if bool(allowed.all()) else torch.where(allowed, 0.0, float("-inf"))
                chunks.append((base_k[..., c0:c1, :], base_v[..., c0:c1, :], mask))
        o, l = ref_walk(C, q, chunks)
        out[name] = {"digest": np.bytes_(I.digest(q, k, v)),
                     "out_qdtype": res.float().numpy().astype(np.float32),
                     "out": o.numpy().astype(np.float32), "lse": l.numpy().astype(np.float32)}
    return out


def gen_config1(C) -> dict:
    """The fp32 CPU-runnable decode case (B1, H32/8, D128, 16 chunks of 512),
    hot = chunks {0, 13, 14, 15}, cold = 1..12; walk
    order cold then hot, as compute_attention walks its tiers."""
    q, k, v = I.config1_inputs()
    chunk = 512
    order = list(range(1, 13)) + [0, 13, 14, 15]
    chunks = [(k[..., c * chunk:(c + 1) * chunk, :], v[..., c * chunk:(c + 1) * chunk, :], None)
              for c in order]
    o, l = ref_walk(C, q, chunks, scale=1.0 / math.sqrt(128))
    return {"config1": {"digest": np.bytes_(I.digest(q, k, v)),
                        "order": np.array(order, dtype=np.int64),
                        "out": o[:, :, 0].numpy().astype(np.float32),
                        "lse": l[:, :, 0].numpy().astype(np.float32)}}


def gen_kivi(K) -> dict:
    out = {}
    for name in I.KIVI_CASES:
        x, bits = I.kivi_inputs(name)
        q, s, z = K._quantize_per_group(x, bits=bits, group_size=32, axis=-1)
        dq = K._dequantize_per_group(q, s, z, group_size=32)
        out[name] = {"digest": np.bytes_(I.digest(x)), "codes": q.numpy().astype(np.int8),
                     "scale_bits": bits16(s), "zero_bits": bits16(z), "dq_bits": bits16(dq)}
    return out


def gen_scorer(Q) -> dict:
    out = {}
    for name in I.SCORER_CASES:
        K, q, page, mr, mp = I.scorer_inputs(name)
        cfg = Q.QuestPathDConfig(page_size=page, memory_ratio=mr, min_pages_selected=mp)
        ad = Q._QuestScorerAdapter(cfg)
        ad.observe_keys(0, K)
        scores = ad.score_pages(0, q)
        top = ad.select_hot_pages(0, q)
        kmin, kmax = ad._k_min[0], ad._k_max[0]
        d = {"digest": np.bytes_(I.digest(K, q)), "scores": scores.float().numpy(),
             "topk": top.numpy().astype(np.int64)}
        if K.dtype == torch.bfloat16:
            d["kmin_bits"], d["kmax_bits"] = bits16(kmin), bits16(kmax)
        else:
            d["kmin"], d["kmax"] = kmin.numpy(), kmax.numpy()
        out[name] = d
    return out


def gen_press(A) -> dict:
    """The reference's HALOPress ablation scorer (page-mean keys, closed-form
    attention + recency + sink score, top-k), plus its uniform-random and FIFO
    selections for the same inputs."""
    out = {}
    for name in I.PRESS_CASES:
        K, q, cfg = I.press_inputs(name)
        c = A.AblationScorerConfig(**cfg)
        ad = A.HALOPressScorerAdapter(c)
        ad.observe_keys(0, K)
        top = ad.select_hot_pages(0, q)
        kmean = ad._k_mean[0]
        d = {"digest": np.bytes_(I.digest(K, q)), "topk": top.numpy().astype(np.int64)}
        if K.dtype == torch.bfloat16:
            d["kmean_bits"] = bits16(kmean)
        else:
            d["kmean"] = kmean.numpy()
        for cls, key in ((A.UniformRandomScorerAdapter, "uniform"), (A.FIFOScorerAdapter, "fifo")):
            other = cls(c)
            other.observe_keys(0, K)
            d[key] = other.select_hot_pages(0, q).numpy().astype(np.int64)
        out[name] = d
    return out


def gen_policy(P) -> dict:
    """The reference's ``HALOConfig`` defaults, ``parse_overrides`` and
    ``with_overrides`` results, as ``repr`` strings (exact, JSON-safe)."""
    import dataclasses
    cfg = P.HALOConfig()
    return {
        "defaults": {f.name: repr(getattr(cfg, f.name)) for f in dataclasses.fields(cfg)},
        "parse_overrides": [repr(P.parse_overrides(s)) for s in I.OVERRIDE_CASES],
        "with_overrides": [
            {f.name: repr(getattr(cfg.with_overrides(d), f.name)) for f in dataclasses.fields(cfg)}
            for d in I.WITH_OVERRIDES_CASES],
    }


def run_host_trace(mods, hot_ratio: float) -> dict:
    """HALOCache.update_hotness over HOST_TRACE with a CPU TieredStorage:
    telemetry and the tier directory after every call.  ``mods`` =
    (HALOConfig, HALOScorer, HALODemoter, HALORefetcher, HALOCache,
    MemoryTier, TieredStorage) of either implementation."""
    Cfg, Scorer, Demoter, Refetcher, Cache, Tier, Storage = mods
    tr = I.HOST_TRACE
    cfg = Cfg(**{**I.HOST_CONFIG, "hot_ratio": hot_ratio})
    st = Storage(tiers=[Tier.GPU, Tier.DRAM], num_layers=tr["layers"],
                 num_kv_heads=tr["kv_heads"], head_dim=tr["head_dim"],
                 block_size=cfg.block_size, dtype=torch.float32, device=torch.device("cpu"),
                 max_blocks=tr["max_blocks"])
    cache = Cache(config=cfg, storage=st, scorer=Scorer(cfg), demoter=Demoter(cfg, storage=st),
                  refetcher=Refetcher(cfg, storage=st))
    n_blocks = tr["K"] // cfg.block_size
    out = []
    for step in range(tr["steps"]):
        for layer in range(tr["layers"]):
            cache.update_hotness(layer, I.host_trace_attention(step, layer, tr["K"]))
            out.append({"telemetry": cache.telemetry(),
                        "directory": [st.locate_block(layer=layer, block=b)
                                      for b in range(n_blocks)],
                        "hot": cache._last_hot_indices[layer].tolist()})
        cache.step()
    return {"trace": out}


def gen_host(mods) -> dict:
    """The reference's host control flow: scorer snapshots (score, hot
    sets, jaccard), refetcher predictions, and update_hotness traces."""
    Cfg, Scorer, _, Refetcher = mods[:4]
    cfg = Cfg(**I.HOST_CONFIG)
    sc, rf = Scorer(cfg), Refetcher(cfg, storage=None)
    snaps = []
    for K, step, seed in I.HOST_SCORE_CASES:
        a = I.host_attention(K, seed)
        s = sc.score(a, step=step)
        hot = sc.topk_hot(s)
        snaps.append({"score": [float(x) for x in s.tolist()], "hot": hot.tolist(),
                      "hot_half": sc.topk_hot(s, ratio=0.5).tolist(),
                      "hot_all": sc.topk_hot(s, ratio=1.0).tolist(),
                      "predicted": rf.predict_hot(layer=0, last_hot_indices=hot,
                                                  last_score=s).tolist()})
    jac = [sc.jaccard(torch.tensor(a, dtype=torch.long), torch.tensor(b, dtype=torch.long))
           for a, b in (([], []), ([1, 2, 3], [2, 3, 4]), ([5], [6]), ([0, 1], [0, 1]))]
    return {"snapshots": snaps, "jaccard": jac,
            "trace_quarter": run_host_trace(mods, 0.25)["trace"],
            "trace_identity": run_host_trace(mods, 1.0)["trace"]}


def save_json(name: str, obj: dict) -> None:
    import json
    path = os.path.join(I.HERE, name)
    with open(path, "w") as f:
        json.dump(obj, f, indent=1, sort_keys=True)
        f.write("\n")
    print(f"wrote {path}: {os.path.getsize(path) / 1024:.1f} KiB")


def save(name: str, groups: dict) -> None:
    flat = {f"{case}/{key}": val for case, arrays in groups.items() for key, val in arrays.items()}
    path = os.path.join(I.HERE, name)
    np.savez_compressed(path, **flat)
    print(f"wrote {path}: {os.path.getsize(path) / 1024:.1f} KiB, {len(groups)} cases")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the lzbaclz/HALO checkout")
    ap.add_argument("--only", default="", help="regenerate one file (e.g. press)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    warnings.filterwarnings("ignore")
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    from halo.kv_cache_chunked import HALOCacheChunked as C
    from halo.demoter import HALODemoter
    from halo.memory_tier import MemoryTier, TieredStorage
    from halo.policy import HALOConfig
    from halo.refetcher import HALORefetcher
    from halo.scorer import HALOScorer
    import baselines.kivi_cache as K
    import baselines.quest_path_d as Q
    import baselines.scorer_ablations as A

    import halo.policy as P

    if args.only == "press":
        save("press.npz", gen_press(A))
        return
    from halo.kv_cache import HALOCache as HC
    host_mods = (HALOConfig, HALOScorer, HALODemoter, HALORefetcher, HC, MemoryTier,
                 TieredStorage)
    if args.only == "policy":
        save_json("policy.json", gen_policy(P))
        return
    if args.only == "host":
        save_json("host.json", gen_host(host_mods))
        return

    def make_cache(chunk, H_kv, D, dtype):
        cfg = HALOConfig(hot_ratio=0.25, tiers=("gpu", "dram"))
        st = TieredStorage(tiers=[MemoryTier.GPU, MemoryTier.DRAM], num_layers=1,
                           num_kv_heads=H_kv, head_dim=D, block_size=32, dtype=dtype,
                           device=torch.device("cpu"))
        return C(config=cfg, storage=st, scorer=HALOScorer(cfg),
                 demoter=HALODemoter(cfg, storage=st), refetcher=HALORefetcher(cfg, storage=st),
                 chunk_size=chunk)

    att = {}
    att.update(gen_walk(C))
    att.update(gen_decode(C, make_cache))
    att.update(gen_prefill(C, make_cache))
    save("attention.npz", att)
    save("config1.npz", gen_config1(C))
    save("kivi.npz", gen_kivi(K))
    save("scorer.npz", gen_scorer(Q))
    save("press.npz", gen_press(A))
    save_json("policy.json", gen_policy(P))
    save_json("host.json", gen_host(host_mods))


if __name__ == "__main__":
    main()
