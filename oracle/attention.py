"""CPU oracle: chunked LSE-merge attention (TEST INFRASTRUCTURE ONLY).

A restatement, in torch CPU fp32 ops, of the reference's per-chunk attention
and log-sum-exp merge.  It produces both the attention output and the LSE
(the reference's ``compute_attention`` drops the LSE, so parity on the LSE
needs this walk).  Reference paths are relative to the lzbaclz/HALO root.
"""
from __future__ import annotations

import math
from typing import Iterable, Optional, Sequence

import torch

NEG_INF = float("-inf")


def _logsumexp_lastdim(x: torch.Tensor) -> torch.Tensor:
    """``torch.logsumexp(x, -1)`` restated with its +-inf max guard.

    An all ``-inf`` row yields ``-inf`` (max forced to 0, sum of zeros).
    """
    m = x.amax(dim=-1, keepdim=True)
    m = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    return torch.log(torch.exp(x - m).sum(dim=-1)) + m.squeeze(-1)


def chunk_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                    scale: Optional[float] = None,
                    mask: Optional[torch.Tensor] = None):
    """One chunk's partial attention ``(out, lse)``.

    Follows ``halo/kv_cache_chunked.py:241-276`` (``_chunk_attention``):
    GQA by repeat-interleave of K/V heads (:260-265), fp32 upcast and
    ``q @ k^T * scale`` (:269-270), additive mask (:271-272), natural-log
    LSE (:273), ``exp(qk - lse) @ v`` (:274-275).

    ``mask`` is a boolean "allowed" tensor broadcastable to
    ``(B, H, T_q, T_c)``; disallowed keys get ``-inf`` before the LSE.
    Rows with no allowed key return ``lse = -inf`` and ``out = 0`` (the
    reference produces NaN there, which its merge then discards, :230-237).
    """
    H, H_kv = q.shape[1], k.shape[1]
    if H != H_kv:
        rep = H // H_kv
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    qk = torch.matmul(q.to(torch.float32), k.to(torch.float32).transpose(-1, -2)) * scale
    if mask is not None:
        qk = torch.where(mask, qk, torch.full_like(qk, NEG_INF))
    lse = _logsumexp_lastdim(qk)
    w = torch.exp(qk - lse.unsqueeze(-1))
    w = torch.where(torch.isneginf(lse).unsqueeze(-1), torch.zeros_like(w), w)
    out = torch.matmul(w, v.to(torch.float32))
    return out, lse


def lse_merge(oa: torch.Tensor, la: torch.Tensor, ob: torch.Tensor, lb: torch.Tensor):
    """Two-way LSE merge; follows ``halo/kv_cache_chunked.py:194-239``.

    ``lse = logaddexp(la, lb)``; weights ``exp(l_x - lse)`` forced to 0 where
    ``l_x == -inf`` (:221-227); outputs of ``-inf`` sides zeroed (:230-237).
    """
    oa, ob = oa.to(torch.float32), ob.to(torch.float32)
    la, lb = la.to(torch.float32), lb.to(torch.float32)
    lse = torch.logaddexp(la, lb)
    a_ninf, b_ninf = torch.isneginf(la), torch.isneginf(lb)
    wa = torch.where(a_ninf, torch.zeros_like(la), (la - lse).exp()).unsqueeze(-1)
    wb = torch.where(b_ninf, torch.zeros_like(lb), (lb - lse).exp()).unsqueeze(-1)
    oa = torch.where(a_ninf.unsqueeze(-1), torch.zeros_like(oa), oa)
    ob = torch.where(b_ninf.unsqueeze(-1), torch.zeros_like(ob), ob)
    return wa * oa + wb * ob, lse


def _causal_allowed(B: int, T_q: int, T_c: int, start: int, q_pos) -> torch.Tensor:
    """Allowed-key mask ``start + j <= q_pos[b] + i`` as ``(B, 1, T_q, T_c)``.

    The per-row rule of ``halo/triton_chunked.py:116-119`` (T_q = 1, per-batch
    ``q_pos``) and of ``halo/kv_cache_chunked.py:894-896`` (T_q > 1, one offset).
    """
    qp = torch.as_tensor(q_pos, dtype=torch.int64).reshape(-1)
    if qp.numel() == 1:
        qp = qp.expand(B)
    i = torch.arange(T_q, dtype=torch.int64).view(1, 1, T_q, 1)
    j = torch.arange(T_c, dtype=torch.int64).view(1, 1, 1, T_c)
    return (start + j) <= (qp.view(B, 1, 1, 1) + i)


def chunked_attention(q: torch.Tensor,
                      chunks: Sequence[tuple],
                      *, scale: Optional[float] = None,
                      q_pos=None):
    """Walk a list of ``(k, v, chunk_start, apply_causal)`` chunks; return
    ``(out, lse)`` in fp32 with ``out`` shaped ``(B, H, T_q, D_v)``.

    Chunk semantics follow ``halo/triton_chunked.py:210-267``
    (``triton_chunked_attention``: default ``q_pos = total_T - 1``, an empty
    list gives zeros) and the per-chunk math/merge of the torch loop
    (``halo/kv_cache_chunked.py:900-908``).  ``q`` may be ``(B, H, D)``.
    """
    if q.dim() == 3:
        q = q.unsqueeze(2)
    B, H, T_q, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if not chunks:
        return (torch.zeros(B, H, T_q, D, dtype=torch.float32),
                torch.full((B, H, T_q), NEG_INF, dtype=torch.float32))
    if q_pos is None:
        q_pos = sum(int(c[0].shape[-2]) for c in chunks) - 1
    run_o = run_l = None
    for k, v, start, causal in chunks:
        T_c = k.shape[-2]
        mask = _causal_allowed(B, T_q, T_c, int(start), q_pos) if causal else None
        o, l = chunk_attention(q, k, v, scale=scale, mask=mask)
        if run_o is None:
            run_o, run_l = o, l
        else:
            run_o, run_l = lse_merge(run_o, run_l, o, l)
    return run_o, run_l


def compute_attention(q: torch.Tensor, *, cold_k=None, cold_v=None,
                      gpu_k=None, gpu_v=None, chunk_size: int = 512,
                      scale: Optional[float] = None,
                      query_pos_offset: Optional[int] = None):
    """Cold-then-recent walk of ``HALOCacheChunked.compute_attention``.

    Follows ``halo/kv_cache_chunked.py:765-964``: empty cache gives zeros
    (:834-837); default ``query_pos_offset = T_total - T_q`` (:839-840);
    cold chunks ``[c0, c1)`` in ``chunk_size`` steps (:874-875), skipped when
    no query may see them (:878-883); recent chunks at global offset
    ``T_cold + c0`` (:919-921), skipped when fully masked (:930-931); causal
    masks only when ``T_q > 1`` (:892-898, :925-932).  Returns fp32
    ``(out, lse)``; the reference returns ``out.to(q.dtype)`` and drops lse.
    """
    B, H, T_q, D = q.shape
    T_cold = cold_k.shape[-2] if cold_k is not None else 0
    T_gpu = gpu_k.shape[-2] if (gpu_k is not None and gpu_k.numel() > 0) else 0
    T_total = T_cold + T_gpu
    if T_total == 0:
        return (torch.zeros(B, H, T_q, D, dtype=torch.float32),
                torch.full((B, H, T_q), NEG_INF, dtype=torch.float32))
    if query_pos_offset is None:
        query_pos_offset = T_total - T_q
    chunk_size = max(1, chunk_size)
    chunks = []
    for base_k, base_v, T_part, offset in ((cold_k, cold_v, T_cold, 0),
                                           (gpu_k, gpu_v, T_gpu, T_cold)):
        for c0 in range(0, T_part, chunk_size):
            c1 = min(c0 + chunk_size, T_part)
            g0 = offset + c0
            if T_q > 1 and g0 > query_pos_offset + T_q - 1:
                continue  # no query row may see this chunk
            chunks.append((base_k[..., c0:c1, :], base_v[..., c0:c1, :], g0, T_q > 1))
    return chunked_attention(q, chunks, scale=scale, q_pos=query_pos_offset)


def full_attention_f64(q, k, v, *, scale=None, q_pos=None, keep=None):
    """One-shot attention in float64 (ground truth for tolerance checks).

    Mirrors the one-shot references of the reference tests
    (``tests/test_triton_chunked.py:31-58``, ``tests/test_kv_cache_chunked.py:20-32``).
    ``keep`` is an optional boolean ``(T,)`` mask of attended positions.
    Returns ``(out, lse)`` with ``out`` shaped ``(B, H, T_q, D_v)``.
    """
    if q.dim() == 3:
        q = q.unsqueeze(2)
    B, H, T_q, D = q.shape
    T = k.shape[-2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    rep = H // k.shape[1]
    kk = k.double().repeat_interleave(rep, dim=1)
    vv = v.double().repeat_interleave(rep, dim=1)
    s = torch.matmul(q.double(), kk.transpose(-1, -2)) * scale
    allowed = torch.ones(B, 1, T_q, T, dtype=torch.bool)
    if q_pos is not None:
        allowed &= _causal_allowed(B, T_q, T, 0, q_pos)
    if keep is not None:
        allowed &= keep.view(1, 1, 1, T)
    s = torch.where(allowed, s, torch.full_like(s, NEG_INF))
    lse = torch.logsumexp(s, dim=-1)
    w = torch.exp(s - lse.unsqueeze(-1))
    w = torch.where(torch.isneginf(lse).unsqueeze(-1), torch.zeros_like(w), w)
    return torch.matmul(w, vv), lse


def acc_state_from_chunks(q, chunks, *, scale=None, q_pos=None):
    """The ``(m, l, o)`` running state of ``halo/triton_chunked.py:47-138``
    after folding ``chunks`` in: ``m`` = max scaled score, ``l = sum exp(s-m)``,
    ``o = sum exp(s-m) v`` (unnormalised).  Derived from ``(out, lse)`` via
    ``m = max score`` (computed directly), ``l = exp(lse - m)``, ``o = out * l``.
    """
    if q.dim() == 3:
        q = q.unsqueeze(2)
    B, H, T_q, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out, lse = chunked_attention(q, chunks, scale=scale, q_pos=q_pos)
    m = torch.full((B, H, T_q), NEG_INF, dtype=torch.float32)
    if q_pos is None:
        q_pos = sum(int(c[0].shape[-2]) for c in chunks) - 1
    rep = H // chunks[0][0].shape[1] if chunks else 1
    for k, v, start, causal in chunks:
        s = torch.matmul(q.float(), k.float().repeat_interleave(rep, dim=1).transpose(-1, -2)) * scale
        if causal:
            s = torch.where(_causal_allowed(B, T_q, k.shape[-2], int(start), q_pos), s,
                            torch.full_like(s, NEG_INF))
        m = torch.maximum(m, s.amax(dim=-1))
    l = torch.where(torch.isneginf(m), torch.zeros_like(m), torch.exp(lse - m))
    o = out * l.unsqueeze(-1)
    return m, l, o


__all__ = [
    "chunk_attention", "lse_merge", "chunked_attention", "compute_attention",
    "full_attention_f64", "acc_state_from_chunks",
]
