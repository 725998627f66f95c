"""CPU oracle: Quest chunk-hotness scorer (TEST INFRASTRUCTURE ONLY).

numpy restatement of ``baselines/quest_path_d.py`` (lzbaclz/HALO):
page summaries, GQA mean-pooled upper-bound scores and top-k selection.
bf16 values travel as raw ``uint16`` bit patterns (numpy has no bfloat16).
"""
from __future__ import annotations

import numpy as np


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    """Exact widening of bf16 bit patterns to float32."""
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even narrowing of float32 to bf16 bit patterns
    (NaN kept quiet)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, np.uint16(0x7FC0), r)


def page_summaries(K: np.ndarray, page_size: int):
    """Per-page channel-wise min/max of K.

    Follows ``baselines/quest_path_d.py:125-150`` (``observe_keys``): only
    full pages ``T // page_size`` (:136), ``amin``/``amax`` over the page's
    tokens (:141-142).  ``K`` is ``(B, H_kv, T, D)`` of any ordered dtype
    (uint16 bf16 bits must be widened first); exact.
    """
    B, H_kv, T, D = K.shape
    n_full = T // page_size
    pages = K[:, :, : n_full * page_size, :].reshape(B, H_kv, n_full, page_size, D)
    return pages.min(axis=-2), pages.max(axis=-2)


def gqa_mean_query(q: np.ndarray, H_kv: int, *, dtype: str) -> np.ndarray:
    """GQA mean-pooled query, ``query.view(B,H_kv,G,T_q,D).mean(dim=2)``
    (``baselines/quest_path_d.py:166-172``), evaluated as torch does for
    reduced precision: fp32 sum over the group, one division by G, one
    rounding back to the query dtype.  ``q``: float32 values of the query.
    Returns float32 values of the rounded mean.
    """
    B, H, T_q, D = q.shape
    if H == H_kv:
        return q.astype(np.float32)
    G = H // H_kv
    g = q.astype(np.float32).reshape(B, H_kv, G, T_q, D)
    s = g[:, :, 0]
    for i in range(1, G):
        s = s + g[:, :, i]
    mean = (s / np.float32(G)).astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(mean))
    if dtype == "f16":
        return mean.astype(np.float16).astype(np.float32)
    return mean


def score_pages(q_g: np.ndarray, k_min: np.ndarray, k_max: np.ndarray) -> np.ndarray:
    """Quest upper bound ``sum_d max(q_d*kmin_d, q_d*kmax_d)`` in fp32.

    Follows ``baselines/quest_path_d.py:175-179``.  ``q_g``: (B,H_kv,T_q,D)
    float32; ``k_min/k_max``: (B,H_kv,P,D) float32.  Returns (B,H_kv,T_q,P).
    The channel sum is done in float64 then rounded: the reference's fp32
    summation order is unspecified, so tests compare scores with a relative
    tolerance and indices modulo ties.
    """
    qe = q_g[:, :, :, None, :].astype(np.float32)
    per_d = np.maximum(qe * k_min[:, :, None].astype(np.float32),
                       qe * k_max[:, :, None].astype(np.float32))
    return per_d.astype(np.float64).sum(axis=-1).astype(np.float32)


def select_topk(scores: np.ndarray, k: int, *, exclude=None) -> np.ndarray:
    """``scores.amax(dim=(0,1,2))`` then top-k, largest first.

    Follows ``baselines/quest_path_d.py:197-202``.  ``exclude`` optionally
    lists page indices masked to ``-inf`` first (hot chunks in the tiered
    decode).  Ties are broken by the lower page index.
    """
    per_page = scores.max(axis=(0, 1, 2)).astype(np.float32)
    if exclude is not None and len(exclude):
        per_page = per_page.copy()
        per_page[np.asarray(exclude, dtype=np.int64)] = -np.inf
    k = min(k, per_page.shape[0])
    order = np.lexsort((np.arange(per_page.shape[0]), -per_page.astype(np.float64)))
    return order[:k].astype(np.int64), per_page


def num_hot_pages(P: int, memory_ratio: float, min_pages: int) -> int:
    """``K = max(min_pages, ceil(P / memory_ratio))`` capped at ``P``;
    ``baselines/quest_path_d.py:199-201`` (integer form of the ceiling)."""
    K = max(min_pages, int((P + memory_ratio - 1) // memory_ratio))
    return min(K, P)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values rounded once to ``dtype`` ("bf16", "f16" or "f32")."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x


def page_means(K: np.ndarray, page_size: int, *, dtype: str) -> np.ndarray:
    """Per-page mean key of the HALOPress scorer
    (``baselines/scorer_ablations.py:208-218``, ``new_k.mean(dim=-2)``): an
    fp32 sum over the page's rows taken in row order, one division by the
    page size, one rounding to the key dtype.  (torch sums in its own order;
    results agree with the reference to one unit in the last place.)
    ``K``: (B, H_kv, T, D) float32 values; only full pages count."""
    B, H_kv, T, D = K.shape
    n = T // page_size
    pages = np.asarray(K, dtype=np.float32)[:, :, : n * page_size].reshape(B, H_kv, n, page_size, D)
    s = pages[:, :, :, 0].copy()
    for r in range(1, page_size):
        s = (s + pages[:, :, :, r]).astype(np.float32)
    return round_to(s / np.float32(page_size), dtype)


def press_scores(q_g: np.ndarray, k_mean: np.ndarray, *, alpha: float, beta: float,
                 gamma: float, sink_tokens: int, refresh_window: int,
                 page_size: int) -> np.ndarray:
    """The HALOPress closed-form page score
    (``baselines/scorer_ablations.py:220-262``): the attention proxy
    ``q . K_mean`` (fp32, channel sum in float64 then rounded: the
    reference's order is unspecified), max over (batch, kv-head, query),
    min-max normalised; a recency term ``exp(-(P-1-p)/window)`` normalised by
    its sum and then its max; sink pages (the first ``sink // page + 1``)
    at 1; ``alpha*attn + beta*rec + gamma*sink`` with one fp32 rounding per
    operation.  ``q_g``: (B, H_kv, T_q, D), ``k_mean``: (B, H_kv, P, D),
    float32 values."""
    f32 = np.float32
    qe = q_g[:, :, :, None, :].astype(np.float32)
    attn = (qe * k_mean[:, :, None].astype(np.float32)).astype(np.float64).sum(axis=-1)
    attn = attn.astype(np.float32).max(axis=(0, 1, 2))
    attn = (attn - attn.min()).astype(np.float32)
    if float(attn.max()) > 0.0:
        attn = (attn / attn.max()).astype(np.float32)
    P = attn.shape[0]
    pos = np.arange(P, dtype=np.float32)
    rec = np.exp(-(f32(P - 1) - pos) / f32(max(refresh_window, 1))).astype(np.float32)
    rec = (rec / (rec.astype(np.float64).sum().astype(np.float32) + f32(1e-12))).astype(np.float32)
    rec = (rec / (rec.max() + f32(1e-12))).astype(np.float32)
    sink = np.zeros(P, dtype=np.float32)
    sink[: min(sink_tokens // max(page_size, 1) + 1, P)] = 1.0
    return ((f32(alpha) * attn + f32(beta) * rec).astype(np.float32) + f32(gamma) * sink).astype(np.float32)


def topk_sorted(score: np.ndarray, k: int) -> np.ndarray:
    """The ``k`` largest pages (ties to the lower index), returned sorted
    ascending as the reference's ``topk(...).indices.sort()`` does."""
    order = np.lexsort((np.arange(score.shape[0]), -score.astype(np.float64)))
    return np.sort(order[:k]).astype(np.int64)


__all__ = ["bf16_bits_to_f32", "f32_to_bf16_bits", "page_summaries",
           "gqa_mean_query", "score_pages", "select_topk", "num_hot_pages", "round_to",
           "page_means", "press_scores", "topk_sorted"]
