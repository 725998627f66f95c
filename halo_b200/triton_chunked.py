"""Name-compatible replacement of ``halo/triton_chunked.py`` (lzbaclz/HALO).

Same functions, arguments and shapes as the reference module's ``__all__``
(:493-501), backed by the sm_100a split-KV + LSE-merge kernels instead of
Triton (there is no Triton here; the module keeps its name so existing
imports keep working).  ``HAS_TRITON`` reports whether the kernel library is
usable, which is what callers of the reference test before dispatching.

Differences that only help: ``triton_chunked_attention`` runs every chunk in
ONE split-KV launch plus one merge launch (the reference launches once per
chunk and recompiles per chunk offset, :52); the streamed and single-launch
variants copy cold chunks with one pitched DMA each on a side stream.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from halo_b200 import ops


def _kernels_available() -> bool:
    try:
        from halo_b200 import _lib
        _lib.lib()
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_TRITON = _kernels_available()


def init_acc(*, B: int, H: int, D_v: int, device, dtype=torch.float32):
    """Fresh running state ``m=-inf (B, H)``, ``l=0 (B, H)``, ``o=0 (B, H, D_v)``
    (``halo/triton_chunked.py:141-148``)."""
    return (torch.full((B, H), float("-inf"), device=device, dtype=dtype),
            torch.zeros((B, H), device=device, dtype=dtype),
            torch.zeros((B, H, D_v), device=device, dtype=dtype))


def update_chunk(*, q, k, v, m, l, o, scale: float, chunk_start: int, q_pos,
                 apply_causal: bool, block_n: int = 64) -> None:
    """Fold one ``(B, H_kv, T_c, D)`` chunk into the running ``(m, l, o)``
    state in place (``halo/triton_chunked.py:151-192``).  ``q``: ``(B, H, D)``.
    Raises ``RuntimeError`` without the kernels, ``AssertionError`` on shape
    mismatch, like the reference."""
    if not HAS_TRITON:
        raise RuntimeError("halo_b200 kernels not available (needs CUDA and libhalo_sm100.so)")
    assert q.dim() == 3, f"expected q (B, H, D), got {q.shape}"
    B, H, D = q.shape
    H_kv, T_c, D_v = k.shape[1], k.shape[2], v.shape[-1]
    assert k.shape == (B, H_kv, T_c, D), f"k shape {k.shape}"
    assert v.shape == (B, H_kv, T_c, D_v), f"v shape {v.shape}"
    qp = q_pos if (q_pos is None or q_pos.is_cuda) else q_pos.to(q.device)
    ops.accumulate_decode(q, [(k, v, chunk_start, apply_causal)], m, l, o, scale=scale, q_pos=qp)


def finalize(*, m, l, o, out_dtype):
    """``o / l`` with zeros where ``l == 0`` (every key masked), cast to
    ``out_dtype`` (``halo/triton_chunked.py:195-207``)."""
    safe = torch.where(l > 0, l, torch.ones_like(l))
    return (o / safe.unsqueeze(-1)).to(out_dtype)


def _q3(q):
    if q.dim() == 4:
        assert q.shape[2] == 1, f"decode path supports T_q=1 only; got {q.shape}"
        return q.squeeze(2)
    return q


def triton_chunked_attention(q, chunks, *, scale: Optional[float] = None, q_pos=None,
                             block_n: int = 64):
    """Attention over ``[(k, v, chunk_start, apply_causal), ...]`` GPU chunks;
    returns ``(B, H, 1, D_v)`` in ``q.dtype`` (``halo/triton_chunked.py:210-267``).
    Default ``q_pos = total_T - 1``; an empty list gives zeros."""
    q3 = _q3(q)
    B, H, D = q3.shape
    if not chunks:
        return torch.zeros(B, H, 1, D, device=q.device, dtype=q.dtype)
    if q_pos is None:
        total = sum(int(c[0].shape[-2]) for c in chunks)
        q_pos = torch.full((B,), total - 1, dtype=torch.int64, device=q.device)
    out, _ = ops.chunked_decode(q3, list(chunks), scale=scale, q_pos=q_pos, out_dtype=q.dtype)
    return out.unsqueeze(2)


def _copy_to(dst, src, stream):
    from halo_b200.kv_cache_chunked import _copy_rows
    try:
        _copy_rows(dst, src, stream)
    except ValueError:   # not pitchable: let torch stage it
        with torch.cuda.stream(stream):
            dst.copy_(src, non_blocking=True)


def triton_chunked_attention_streamed(q, cold_chunks_host, hot_chunks_gpu, *,
                                      scale: Optional[float] = None, q_pos, block_n: int = 64,
                                      n_buffers: int = 2):
    """Cold host chunks ``[(k, v, start), ...]`` streamed to HBM on a side
    stream (``n_buffers`` staging slots) while earlier chunks are attended;
    hot GPU chunks attended in place (``halo/triton_chunked.py:270-362``).
    Returns ``(B, H, 1, D_v)`` in ``q.dtype``."""
    q3 = _q3(q).contiguous()
    B, H, D = q3.shape
    first = next(iter([c for c in cold_chunks_host] + [c for c in hot_chunks_gpu]), None)
    if first is None:
        return torch.zeros(B, H, 1, D, device=q.device, dtype=q.dtype)
    D_v = first[1].shape[-1]
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    qp = q_pos.to(device=q.device, dtype=torch.int64)
    m, l, o = init_acc(B=B, H=H, D_v=D_v, device=q.device)
    if hot_chunks_gpu:
        ops.accumulate_decode(q3, [(k, v, s, True) for (k, v, s) in hot_chunks_gpu], m, l, o,
                              scale=scale, q_pos=qp)
    if cold_chunks_host:
        cur = torch.cuda.current_stream()
        cs = torch.cuda.Stream()
        cs.wait_stream(cur)
        slots, ready, free = [None] * n_buffers, [torch.cuda.Event() for _ in range(n_buffers)], \
            [torch.cuda.Event() for _ in range(n_buffers)]
        for i, (kh, vh, start) in enumerate(cold_chunks_host):
            s = i % n_buffers
            if slots[s] is None or slots[s][0].shape != kh.shape:
                slots[s] = (torch.empty(kh.shape, dtype=kh.dtype, device=q.device),
                            torch.empty(vh.shape, dtype=vh.dtype, device=q.device))
                cs.wait_stream(cur)
                for t in slots[s]:
                    t.record_stream(cs)
            if i >= n_buffers:
                cs.wait_event(free[s])
            _copy_to(slots[s][0], kh, cs)
            _copy_to(slots[s][1], vh, cs)
            ready[s].record(cs)
            cur.wait_event(ready[s])
            ops.accumulate_decode(q3, [(slots[s][0], slots[s][1], start, True)], m, l, o,
                                  scale=scale, q_pos=qp)
            free[s].record(cur)
    return finalize(m=m, l=l, o=o, out_dtype=q.dtype).unsqueeze(2)


def triton_chunked_attention_single_launch(q, cold_k_host, cold_v_host, hot_k_gpu, hot_v_gpu, *,
                                           scale: Optional[float] = None, q_pos,
                                           block_n: int = 64, apply_causal: bool = True):
    """One copy of the whole cold prefix to HBM (side stream, one pitched DMA
    per tensor) and one attention launch over cold + hot
    (``halo/triton_chunked.py:365-490``).  Returns ``(B, H, 1, D_v)``."""
    q3 = _q3(q).contiguous()
    B, H, D = q3.shape
    ref = next((t for t in (cold_v_host, hot_v_gpu) if t is not None and t.shape[-2] > 0), None)
    if ref is None:
        return torch.zeros(B, H, 1, D, device=q.device, dtype=q.dtype)
    T_cold = cold_k_host.shape[-2] if cold_k_host is not None else 0
    T_hot = hot_k_gpu.shape[-2] if hot_k_gpu is not None else 0
    qp = q_pos.to(device=q.device, dtype=torch.int64)
    chunks = []
    if T_cold > 0:
        cs = torch.cuda.Stream()
        kc = torch.empty(cold_k_host.shape, dtype=cold_k_host.dtype, device=q.device)
        vc = torch.empty(cold_v_host.shape, dtype=cold_v_host.dtype, device=q.device)
        cs.wait_stream(torch.cuda.current_stream())
        _copy_to(kc, cold_k_host, cs)
        _copy_to(vc, cold_v_host, cs)
        torch.cuda.current_stream().wait_stream(cs)
        kc.record_stream(cs)
        vc.record_stream(cs)
        chunks.append((kc, vc, 0, apply_causal))
    if T_hot > 0:
        chunks.append((hot_k_gpu, hot_v_gpu, T_cold, apply_causal))
    out, _ = ops.chunked_decode(q3, chunks, scale=scale, q_pos=qp, out_dtype=q.dtype)
    return out.unsqueeze(2)


__all__ = [
    "HAS_TRITON",
    "init_acc",
    "update_chunk",
    "finalize",
    "triton_chunked_attention",
    "triton_chunked_attention_streamed",
    "triton_chunked_attention_single_launch",
]
