"""ctypes binding of ``libhalo_sm100.so`` (declared in ``include/halo_b200.h``).

The library is required: importing an op without it raises ``HaloError``.
There is no CPU fallback anywhere in the package.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import threading

import torch  # noqa: F401  -- loads the CUDA runtime the library shares with torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libhalo_sm100.so")

HALO_OK = 0
HALO_ERR_INVALID_ARG = -1
HALO_ERR_UNSUPPORTED = -2
HALO_ERR_MISALIGNED = -3
HALO_ERR_CUDA = -4
HALO_ERR_TIMEOUT = -5
HALO_ERR_WORKSPACE = -6
HALO_ERR_SPLIT = -7

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
MERGE_FINALIZE, MERGE_ACCUMULATE = 0, 1

_TORCH_TO_HALO = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}


class HaloError(RuntimeError):
    """A libhalo_sm100 call failed (status code in ``.code``)."""

    def __init__(self, msg: str, code: int = 0):
        super().__init__(msg)
        self.code = code


def halo_dtype(dt: torch.dtype) -> int:
    try:
        return _TORCH_TO_HALO[dt]
    except KeyError:
        raise HaloError(f"unsupported dtype {dt}", HALO_ERR_UNSUPPORTED) from None


class KVChunk(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("k_stride_b", ctypes.c_int64), ("k_stride_h", ctypes.c_int64),
                ("k_stride_t", ctypes.c_int64),
                ("v_stride_b", ctypes.c_int64), ("v_stride_h", ctypes.c_int64),
                ("v_stride_t", ctypes.c_int64),
                ("start", ctypes.c_int64), ("len", ctypes.c_int32), ("causal", ctypes.c_int32)]


class DecodeProblem(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int32), ("H", ctypes.c_int32), ("H_kv", ctypes.c_int32),
                ("D", ctypes.c_int32), ("Dv", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("q", ctypes.c_void_p), ("q_stride_b", ctypes.c_int64),
                ("q_stride_h", ctypes.c_int64), ("q_pos", ctypes.c_void_p),
                ("scale", ctypes.c_float), ("max_split_rows", ctypes.c_int32),
                ("event_begin", ctypes.c_void_p), ("event_end", ctypes.c_void_p)]


class MergeArgs(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
                ("out", ctypes.c_void_p), ("out_stride_b", ctypes.c_int64),
                ("out_stride_h", ctypes.c_int64), ("lse", ctypes.c_void_p),
                ("m", ctypes.c_void_p), ("l", ctypes.c_void_p), ("o", ctypes.c_void_p)]


class KiviTensor(ctypes.Structure):
    _fields_ = [("codes", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("zero", ctypes.c_void_p),
                ("codes_stride_b", ctypes.c_int64), ("codes_stride_h", ctypes.c_int64),
                ("sz_stride_b", ctypes.c_int64), ("sz_stride_h", ctypes.c_int64),
                ("t_cap", ctypes.c_int64)]


class PrefillProblem(ctypes.Structure):
    _fields_ = [("B", ctypes.c_int32), ("H", ctypes.c_int32), ("H_kv", ctypes.c_int32),
                ("T_q", ctypes.c_int32), ("D", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("q", ctypes.c_void_p), ("q_stride_b", ctypes.c_int64),
                ("q_stride_h", ctypes.c_int64), ("q_stride_t", ctypes.c_int64),
                ("q_pos0", ctypes.c_int64), ("scale", ctypes.c_float),
                ("event_begin", ctypes.c_void_p), ("event_end", ctypes.c_void_p)]


class PrefillOut(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
                ("out", ctypes.c_void_p), ("out_stride_b", ctypes.c_int64),
                ("out_stride_h", ctypes.c_int64), ("out_stride_t", ctypes.c_int64),
                ("lse", ctypes.c_void_p), ("m", ctypes.c_void_p), ("l", ctypes.c_void_p),
                ("o", ctypes.c_void_p)]


# name -> (restype, argtypes); must match include/halo_b200.h
SIGNATURES = {
    "halo_decode_workspace_bytes": (ctypes.c_int64, [ctypes.POINTER(DecodeProblem),
                                                     ctypes.POINTER(KVChunk), ctypes.c_int32]),
    "halo_chunked_decode": (ctypes.c_int32, [ctypes.POINTER(DecodeProblem), ctypes.POINTER(KVChunk),
                                             ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                                             ctypes.POINTER(MergeArgs), ctypes.c_void_p]),
    "halo_chunked_decode_noalloc": (ctypes.c_int32, [ctypes.POINTER(DecodeProblem),
                                                     ctypes.POINTER(KVChunk), ctypes.c_int32,
                                                     ctypes.POINTER(MergeArgs), ctypes.c_void_p]),
    "halo_lse_merge": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_int64,
                                        ctypes.POINTER(MergeArgs), ctypes.c_void_p]),
    "halo_kivi_quantize": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                            ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]),
    "halo_kivi_dequantize": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]),
    "halo_kivi_decode_workspace_bytes": (ctypes.c_int64, [ctypes.POINTER(DecodeProblem),
                                                          ctypes.c_int32]),
    "halo_kivi_decode": (ctypes.c_int32, [ctypes.POINTER(DecodeProblem), ctypes.POINTER(KiviTensor),
                                          ctypes.POINTER(KiviTensor), ctypes.c_int32, ctypes.c_int32,
                                          ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
                                          ctypes.c_int64, ctypes.POINTER(MergeArgs),
                                          ctypes.c_void_p]),
    "halo_page_summary": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                           ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                           ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_void_p]),
    "halo_page_score_topk": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_void_p]),
    "halo_page_mean": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_void_p]),
    "halo_page_press_topk": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                              ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                              ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                              ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_void_p]),
    "halo_copy2d_async": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                           ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_void_p]),
    "halo_last_error_string": (ctypes.c_char_p, []),
    "halo_device_error": (ctypes.c_int32, [ctypes.POINTER(ctypes.c_int32), ctypes.c_int32]),
    "halo_prefill_attention": (ctypes.c_int32, [ctypes.POINTER(PrefillProblem),
                                                ctypes.POINTER(KVChunk), ctypes.c_int32,
                                                ctypes.POINTER(PrefillOut), ctypes.c_void_p]),
    "halo_prefill_workspace_bytes": (ctypes.c_int64, [ctypes.POINTER(PrefillProblem),
                                                      ctypes.POINTER(KVChunk), ctypes.c_int32]),
    "halo_prefill_attention_ws": (ctypes.c_int32, [ctypes.POINTER(PrefillProblem),
                                                   ctypes.POINTER(KVChunk), ctypes.c_int32,
                                                   ctypes.POINTER(PrefillOut), ctypes.c_void_p,
                                                   ctypes.c_int64, ctypes.c_void_p]),
    "halo_chunked_decode_partials": (ctypes.c_int32, [ctypes.POINTER(DecodeProblem),
                                                      ctypes.POINTER(KVChunk), ctypes.c_int32,
                                                      ctypes.c_void_p, ctypes.c_int64,
                                                      ctypes.POINTER(ctypes.c_int32),
                                                      ctypes.POINTER(ctypes.c_int64),
                                                      ctypes.c_void_p]),
    "halo_exchange_bytes": (ctypes.c_int64, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "halo_ipc_alloc": (ctypes.c_int32, [ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p),
                                        ctypes.c_void_p]),
    "halo_ipc_open": (ctypes.c_int32, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "halo_ipc_close": (ctypes.c_int32, [ctypes.c_void_p]),
    "halo_ipc_free": (ctypes.c_int32, [ctypes.c_void_p]),
    "halo_sharded_merge": (ctypes.c_int32, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                            ctypes.c_int32,
                                            ctypes.POINTER(ctypes.c_void_p), ctypes.c_int32,
                                            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_void_p, ctypes.c_void_p]),
    "halo_sharded_decode": (ctypes.c_int32, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                             ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
                                             ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p),
                                             ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                                             ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]),
    "halo_version": (ctypes.c_int32, []),
    "halo_launch_count": (ctypes.c_uint64, []),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load ``libhalo_sm100.so`` once; raise ``HaloError`` if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise HaloError(f"{LIB_PATH} not built; run `python -m halo_b200.build`")
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != HALO_OK:
        msg = lib().halo_last_error_string()
        raise HaloError(f"{what} failed ({rc}): {msg.decode() if msg else ''}", rc)


def device_error(clear: bool = True) -> int:
    """Read (and clear) the device error word; 0 or a HALO_ERR_* code."""
    code = ctypes.c_int32(0)
    check(lib().halo_device_error(ctypes.byref(code), int(clear)), "halo_device_error")
    return code.value


def launch_count() -> int:
    """Kernels this library has launched in this process."""
    return int(lib().halo_launch_count())


# The raw cudaStream_t of a device's current stream without building a
# torch.cuda.Stream object (~0.3 us against ~2.5 us of host time per call).
_raw_current_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: torch.device) -> int:
    """The raw handle of ``device``'s current CUDA stream."""
    if _raw_current_stream is not None:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return int(_raw_current_stream(idx))
    return torch.cuda.current_stream(device).cuda_stream


def on_device(device: torch.device):
    """``torch.cuda.device(device)``, or a no-op context when ``device`` is
    already the current device (entering the torch context costs ~2 us of
    host time, as much as the rest of a small decode call's set-up)."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)
