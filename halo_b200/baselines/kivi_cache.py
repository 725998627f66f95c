"""KIVI 2/4/8-bit KV cache on the B200 kernels.

Mirrors ``baselines/kivi_cache.py`` of lzbaclz/HALO (:44-226):
``_quantize_per_group`` / ``_dequantize_per_group`` (bit-exact, in
``libhalo_sm100.so``), ``KIVICache`` (recent rows kept in 16-bit, older rows
quantised in groups of ``group_size`` along head_dim) and ``wrap_with_kivi``.

Differences that only help:

* codes are stored PACKED (8/bits per byte) with 16-bit scale/zero per group
  in HBM, appended in place (the reference keeps int8 codes and re-concatenates
  every update);
* ``compute_attention`` attends the packed prefix with the fused
  dequantise-and-attend kernel (``halo_kivi_decode``) and the recent rows with
  the split-KV kernel, merged by LSE -- no per-step full dequantisation;
* ``update`` still returns the dequantised ``(K, V)`` (the reference contract,
  :187-195) unless ``fused_attention=True``, in which case it returns the
  recent rows and attention must go through ``compute_attention``.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from halo_b200 import _lib as L
from halo_b200 import ops

try:
    from transformers.cache_utils import DynamicCache as _BaseCache
except Exception:  # pragma: no cover
    class _BaseCache:  # type: ignore[no-redef]
        def __init__(self):
            pass


def _check_cuda(t, name):
    if not t.is_cuda:
        raise L.HaloError(f"{name} must be a CUDA tensor (no CPU path)", L.HALO_ERR_INVALID_ARG)


def quantize_packed(x: torch.Tensor, *, bits: int, group_size: int):
    """Quantise ``x (B, H, T, D)`` (fp16/bf16, CUDA) along head_dim.  Returns
    ``(codes uint8 (B, H, T, D*bits/8), scale (B, H, T, D/group), zero)``."""
    _check_cuda(x, "x")
    B, H, T, D = x.shape
    x = x if x.stride(-1) == 1 else x.contiguous()
    codes = torch.empty(B, H, T, D * bits // 8, dtype=torch.uint8, device=x.device)
    scale = torch.empty(B, H, T, D // group_size, dtype=x.dtype, device=x.device)
    zero = torch.empty_like(scale)
    _quant_into(x, codes, scale, zero, bits, group_size)
    return codes, scale, zero


def _quant_into(x, codes, scale, zero, bits, group):
    B, H, T, D = x.shape
    with torch.cuda.device(x.device):
        rc = L.lib().halo_kivi_quantize(
            x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), B, H, T, D,
            L.halo_dtype(x.dtype), bits, group, codes.data_ptr(), codes.stride(0),
            codes.stride(1), codes.stride(2), scale.data_ptr(), zero.data_ptr(), scale.stride(0),
            scale.stride(1), scale.stride(2), L.stream_handle(x.device))
    L.check(rc, "halo_kivi_quantize")


def dequantize_packed(codes, scale, zero, *, bits: int, group_size: int, out=None):
    """Inverse of :func:`quantize_packed` (``rnd(fl32(q*s) + z)``)."""
    _check_cuda(codes, "codes")
    B, H, T, CB = codes.shape
    D = CB * 8 // bits
    if out is None:
        out = torch.empty(B, H, T, D, dtype=scale.dtype, device=codes.device)
    with torch.cuda.device(codes.device):
        rc = L.lib().halo_kivi_dequantize(
            codes.data_ptr(), codes.stride(0), codes.stride(1), codes.stride(2), scale.data_ptr(),
            zero.data_ptr(), scale.stride(0), scale.stride(1), scale.stride(2), B, H, T, D,
            L.halo_dtype(scale.dtype), bits, group_size, out.data_ptr(), out.stride(0),
            out.stride(1), out.stride(2), L.stream_handle(codes.device))
    L.check(rc, "halo_kivi_dequantize")
    return out


def unpack_codes(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """Packed codes ``(..., D*bits/8)`` -> uint8 codes ``(..., D)``.  4/8
    bits: code ``i`` at byte ``i*bits/8``, bit ``(i*bits)%8``.  2 bits: 16
    codes per little-endian 32-bit word, code ``i`` at word ``i/16``, bit
    ``16*(e&1) + 2*(e>>1)`` with ``e = i%16`` (the decoder's pair layout:
    codes 2q and 2q+1 share bit 2q of the word's two halves)."""
    lead, nb = codes.shape[:-1], codes.shape[-1]
    if bits == 2:
        e = torch.arange(16, device=codes.device)
        pos = 16 * (e & 1) + 2 * (e >> 1)
        byte, shift = (pos // 8), (pos % 8).to(torch.uint8)
        w = codes.reshape(*lead, nb // 4, 4)
        return ((w[..., byte] >> shift) & 3).reshape(*lead, nb * 4)
    per = 8 // bits
    c = codes.unsqueeze(-1).expand(*codes.shape, per)
    shifts = torch.arange(per, device=codes.device, dtype=torch.uint8) * bits
    return ((c >> shifts) & ((1 << bits) - 1)).reshape(*lead, nb * per)


def _quantize_per_group(x, *, bits: int, group_size: int, axis: int):
    """Reference-shaped quantisation (``baselines/kivi_cache.py:44-69``):
    returns unpacked int8 codes ``(..., D/g, g)`` and scale/zero
    ``(..., D/g, 1)`` in x's dtype, bit-exact."""
    assert axis == -1, "current implementation supports axis=-1 only"
    shp = x.shape
    x4 = x.reshape(-1, 1, shp[-2] if x.dim() > 1 else 1, shp[-1]) if x.dim() != 4 else x
    codes, scale, zero = quantize_packed(x4, bits=bits, group_size=group_size)
    q = unpack_codes(codes, bits)
    g = shp[-1] // group_size
    return (q.to(torch.int8).reshape(*shp[:-1], g, group_size),
            scale.reshape(*shp[:-1], g, 1), zero.reshape(*shp[:-1], g, 1))


def _dequantize_per_group(q, scale, zero, *, group_size: int):
    """Reference-shaped dequantisation (``baselines/kivi_cache.py:72-78``):
    unpacked codes ``(..., D/g, g)`` are already a valid 8-bit packing."""
    g = q.shape[-2]
    D = g * group_size
    lead = q.shape[:-2]
    codes = q.reshape(1, 1, -1, D).to(torch.uint8).contiguous()
    s = scale.reshape(1, 1, -1, g).contiguous()
    z = zero.reshape(1, 1, -1, g).contiguous()
    out = dequantize_packed(codes, s, z, bits=8, group_size=group_size)
    return out.reshape(*lead, D)


class _Packed:
    """One layer's packed K or V: rows [0, T) valid, capacity a multiple of 64."""

    def __init__(self, B, H, D, dtype, device, bits, group):
        self.B, self.H, self.D, self.dtype, self.dev = B, H, D, dtype, device
        self.bits, self.group = bits, group
        self.T = 0
        self.codes = self.scale = self.zero = None
        self._view = None       # C-ABI description of the storage; reset when it moves

    def reserve(self, rows: int) -> None:
        cap = 0 if self.codes is None else self.codes.shape[2]
        if self.T + rows <= cap:
            return
        new_cap = max(self.T + rows, 2 * cap, 256)
        new_cap = (new_cap + 63) // 64 * 64
        codes = torch.zeros(self.B, self.H, new_cap, self.D * self.bits // 8, dtype=torch.uint8,
                            device=self.dev)
        scale = torch.zeros(self.B, self.H, new_cap, self.D // self.group, dtype=self.dtype,
                            device=self.dev)
        zero = torch.zeros_like(scale)
        if self.T:
            codes[:, :, :self.T].copy_(self.codes[:, :, :self.T])
            scale[:, :, :self.T].copy_(self.scale[:, :, :self.T])
            zero[:, :, :self.T].copy_(self.zero[:, :, :self.T])
        self.codes, self.scale, self.zero = codes, scale, zero
        self._view = None

    def append(self, x) -> None:
        n = x.shape[2]
        self.reserve(n)
        _quant_into(x, self.codes[:, :, self.T:self.T + n], self.scale[:, :, self.T:self.T + n],
                    self.zero[:, :, self.T:self.T + n], self.bits, self.group)
        self.T += n

    def dequantized(self):
        return dequantize_packed(self.codes[:, :, :self.T], self.scale[:, :, :self.T],
                                 self.zero[:, :, :self.T], bits=self.bits, group_size=self.group)

    def view(self) -> L.KiviTensor:
        """The storage's C-ABI description (pointers, strides, capacity); it
        stays valid until ``reserve`` moves the storage."""
        if self._view is not None:
            return self._view
        t = self._view = L.KiviTensor()
        t.codes, t.scale, t.zero = self.codes.data_ptr(), self.scale.data_ptr(), self.zero.data_ptr()
        t.codes_stride_b, t.codes_stride_h = self.codes.stride(0), self.codes.stride(1)
        t.sz_stride_b, t.sz_stride_h = self.scale.stride(0), self.scale.stride(1)
        t.t_cap = self.codes.shape[2]
        return t


class KIVICache(_BaseCache):
    """KV cache with KIVI-style 2/4/8-bit quantisation (per-group along
    head_dim for K and V, as the reference code does) and a 16-bit recent
    buffer of ``residual_length`` rows."""

    def __init__(self, *, bits: int = 2, group_size: int = 32, residual_length: int = 32,
                 fused_attention: bool = False) -> None:
        super().__init__()
        self.bits = bits
        self.group_size = group_size
        self.residual_length = residual_length
        self.fused_attention = fused_attention
        self._k_recent: list = []
        self._v_recent: list = []
        self._k_quant: list = []
        self._v_quant: list = []
        self._n_seen: list = []
        self._ones_cache: dict = {}
        self._recent_tables: dict = {}   # layer -> ChunkTable of its recent rows
        # fp32 (out, lse) of the packed prefix per (device, stream, B, H, D):
        # written and consumed on that stream within one call, so stream
        # order makes reuse across calls and layers safe
        self._prefix_state: dict = {}

    @classmethod
    def from_memory_ratio(cls, *, memory_ratio: int, **kw) -> "KIVICache":
        return cls(bits=max(16 // memory_ratio, 2), **kw)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        if layer_idx >= len(self._n_seen):
            return 0
        rec = self._k_recent[layer_idx]
        return self._n_seen[layer_idx] + (rec.shape[-2] if rec is not None else 0)

    def update(self, key_states, value_states, layer_idx, *args, **kwargs):
        """Append; quantise the overflow beyond ``residual_length`` rounded
        down to a multiple of ``group_size`` rows (``:121-195``)."""
        _check_cuda(key_states, "key_states")
        while len(self._k_recent) <= layer_idx:
            self._k_recent.append(None)
            self._v_recent.append(None)
            self._k_quant.append(None)
            self._v_quant.append(None)
            self._n_seen.append(0)
        kr, vr = self._k_recent[layer_idx], self._v_recent[layer_idx]
        kr = key_states if kr is None else torch.cat([kr, key_states], dim=-2)
        vr = value_states if vr is None else torch.cat([vr, value_states], dim=-2)
        overflow = kr.shape[-2] - self.residual_length
        if overflow > 0:
            oq = (overflow // self.group_size) * self.group_size
            if oq > 0:
                if self._k_quant[layer_idx] is None:
                    B, H, _, D = kr.shape
                    self._k_quant[layer_idx] = _Packed(B, H, D, kr.dtype, kr.device, self.bits,
                                                       self.group_size)
                    self._v_quant[layer_idx] = _Packed(B, H, vr.shape[-1], vr.dtype, vr.device,
                                                       self.bits, self.group_size)
                self._k_quant[layer_idx].append(kr[..., :oq, :])
                self._v_quant[layer_idx].append(vr[..., :oq, :])
                self._n_seen[layer_idx] += oq
                kr = kr[..., oq:, :].contiguous()
                vr = vr[..., oq:, :].contiguous()
        self._k_recent[layer_idx], self._v_recent[layer_idx] = kr, vr
        self._recent_tables.pop(layer_idx, None)
        if self.fused_attention or self._k_quant[layer_idx] is None:
            return kr, vr
        return (torch.cat([self._k_quant[layer_idx].dequantized(), kr], dim=-2),
                torch.cat([self._v_quant[layer_idx].dequantized(), vr], dim=-2))

    def compute_attention(self, q, *, layer_idx: int, scaling: Optional[float] = None,
                          events: Optional[tuple] = None):
        """Attention of ``q (B, H, T_q, D)`` over the quantised prefix (its
        dequantised values, as the reference attends them) plus the recent
        rows; decode (T_q = 1) runs the fused packed kernel.  ``events =
        (begin, end)`` (raw ``cudaEvent_t``) bracket that kernel (profiling)."""
        B, H, T_q, D = q.shape
        scale = float(scaling) if scaling is not None else 1.0 / math.sqrt(D)
        kq, vq = self._k_quant[layer_idx], self._v_quant[layer_idx]
        kr, vr = self._k_recent[layer_idx], self._v_recent[layer_idx]
        T_quant = kq.T if kq is not None else 0
        if T_q > 1:
            chunks = []
            if T_quant:
                chunks.append((kq.dequantized(), vq.dequantized(), 0, True))
            if kr is not None and kr.shape[-2]:
                chunks.append((kr, vr, T_quant, True))
            T_total = T_quant + (kr.shape[-2] if kr is not None else 0)
            out, _ = ops.multi_query_attention(q, chunks, scale=scale,
                                               query_pos_offset=T_total - T_q)
            return out
        q3 = q.squeeze(2).contiguous()
        dev = q.device
        recent = None
        if kr is not None and kr.shape[-2]:
            recent = self._recent_tables.get(layer_idx)
            if recent is None:
                recent = self._recent_tables[layer_idx] = ops.ChunkTable([(kr, vr, T_quant, False)])
        prior = None
        if T_quant:
            # The prefix's normalised (out, lse) is a running state with l = 1.
            key = (dev.index, L.stream_handle(dev), B, H, D)
            st = self._prefix_state.get(key)
            if st is None:
                st = self._prefix_state[key] = (
                    torch.empty(B, H, D, dtype=torch.float32, device=dev),
                    torch.empty(B, H, dtype=torch.float32, device=dev))
            o32, lse = st
            kivi_decode(q3, kq, vq, T_quant, self.bits, scale=scale, out=o32, lse=lse,
                        events=events)
            if recent is None:
                return o32.to(q.dtype, copy=True).unsqueeze(2)
            prior = (lse, self._ones(B, H, dev), o32)
        out, _ = ops.chunked_decode(q3, recent if recent is not None else [], scale=scale,
                                    prior=prior, want_lse=False)
        return out.unsqueeze(2)

    def _ones(self, B: int, H: int, dev) -> torch.Tensor:
        key = (B, H, dev.index)
        t = self._ones_cache.get(key)
        if t is None:
            t = self._ones_cache[key] = torch.ones(B, H, dtype=torch.float32, device=dev)
        return t

    def reset(self) -> None:
        self._k_recent.clear()
        self._v_recent.clear()
        self._k_quant.clear()
        self._v_quant.clear()
        self._n_seen.clear()
        self._recent_tables.clear()


def kivi_decode(q3, kq: _Packed, vq: _Packed, rows: int, bits: int, *, scale: float,
                state=None, out=None, lse=None, events=None):
    """Fused packed decode over ``rows`` quantised rows.  ``state=(m, l, o)``
    accumulates into running fp32 state; otherwise returns ``(out, lse)``."""
    B, H, D = q3.shape
    p = ops._problem(q3, kq.H, D, None, scale)
    if events is not None:
        p.event_begin, p.event_end = events
    kt, vt = kq.view(), vq.view()
    lib = L.lib()
    need = lib.halo_kivi_decode_workspace_bytes(ctypes.byref(p), rows)
    if need < 0:
        L.check(int(need), "halo_kivi_decode_workspace_bytes")
    sh = L.stream_handle(q3.device)
    ws = ops.WORKSPACES.get(q3.device, int(need), sh)
    mg = L.MergeArgs()
    if state is not None:
        m, l, o = state
        mg.mode = L.MERGE_ACCUMULATE
        mg.m, mg.l, mg.o = m.data_ptr(), l.data_ptr(), o.data_ptr()
    else:
        out = out if out is not None else torch.empty(B, H, D, dtype=q3.dtype, device=q3.device)
        lse = lse if lse is not None else torch.empty(B, H, dtype=torch.float32, device=q3.device)
        mg.mode = L.MERGE_FINALIZE
        mg.out_dtype = L.halo_dtype(out.dtype)
        mg.out = out.data_ptr()
        mg.out_stride_b, mg.out_stride_h = out.stride(0), out.stride(1)
        mg.lse = lse.data_ptr()
    with L.on_device(q3.device):
        rc = lib.halo_kivi_decode(ctypes.byref(p), ctypes.byref(kt), ctypes.byref(vt), rows, bits, 0,
                                  0, ws.data_ptr(), ws.numel(), ctypes.byref(mg), sh)
    L.check(rc, "halo_kivi_decode")
    return (out, lse) if state is None else None


def wrap_with_kivi(model, *, memory_ratio: int = 4, **kw):
    """Give ``model.generate`` a fresh :class:`KIVICache` per call
    (``baselines/kivi_cache.py:205-226``)."""
    cache = KIVICache.from_memory_ratio(memory_ratio=memory_ratio, **kw)
    if getattr(model, "_kivi_patched", False):
        return model
    original = model.generate

    def kivi_generate(*args, **kwargs):
        cache.reset()
        kwargs.setdefault("past_key_values", cache)
        kwargs.setdefault("use_cache", True)
        return original(*args, **kwargs)

    model.generate = kivi_generate
    model._kivi_patched = True
    model._kivi_cache = cache
    return model


__all__ = ["_quantize_per_group", "_dequantize_per_group", "KIVICache", "wrap_with_kivi",
           "quantize_packed", "dequantize_packed", "unpack_codes", "kivi_decode"]
