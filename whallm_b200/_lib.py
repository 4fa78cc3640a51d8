"""ctypes binding of ``libwhallm_b200.so`` (the C ABI in ``include/whallm_b200.h``).

There is no CPU or PyTorch fallback: if the shared library is missing or a
call fails, an exception is raised.  Tensors cross the boundary as raw device
pointers plus sizes, together with the current CUDA stream of their device.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libwhallm_b200.so")

WM_OK = 0
WM_ERR_INVALID = -1
WM_ERR_UNSUPPORTED = -2
WM_ERR_CUDA = -3
WM_ERR_WORKSPACE = -4

WM_OUT_F32, WM_OUT_BF16 = 0, 1
WM_SCORE_SOFTMAX, WM_SCORE_SIGMOID, WM_SCORE_SQRTSOFTPLUS, WM_SCORE_NONE, WM_SCORE_SOFTMAX_BF16 = 0, 1, 2, 3, 4
WM_UP_GATE, WM_GATE_UP = 0, 1
WKV_FP8_F32_B64, WKV_FP8_UE8M0_B32, WKV_FP4_E4M3_B16, WKV_FP4_UE8M0_B32, WKV_MXFP8_B32, WKV_MXFP4_B32 = range(6)

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> argtypes (restype int unless listed in _RESTYPE)
SIGNATURES = {
    "w_last_error": [],
    "w_abi_version": [],
    "wmxfp4_quantize": [_P, _I64, _I64, _P, _P, _P],
    "wmxfp4_dequantize": [_P, _P, _I64, _I64, _I, _P, _P],
    "wmx_split_e4m3": [_P, _I, _I, _P, _P, _P, _P],
    "wkv_scores_workspace_size": [_I, _I, _I, _I],
    "wmx_linear_workspace_size": [_I, _I, _I],
    "wmx_linear": [_P, _I, _I, _P, _P, _I, _I, _P, _P, _SZ, _P],
    "wkv_mx_scores": [_P, _I, _I, _I, _P, _P, _I, _I, _P, _P, _SZ, _P],
    "wep_ipc_alloc": [_SZ, _P, _P],
    "wep_ipc_open": [_P, _P],
    "wep_ipc_close": [_P],
    "wep_ipc_free": [_P],
    "wep_put_rows": [_I, _P, _P, _P, _P, _I, _P, _I, _I, _P, _P, _P, _P],
    "wep_wait": [_P, _I, _P, _P, _P],
    "wep_sum_rows": [_P, _I, _I, _I, _P, _P, _P],
    "wld_load_expert_layer": [ctypes.c_char_p, _SZ, _I, _I, _P, _P, _P, _P, _SZ, _P],
    "waffine4_quantize": [_P, _I64, _I64, _I, _P, _P, _P, _P],
    "waffine4_dequantize": [_P, _P, _P, _I64, _I64, _I, _I, _P, _P],
    "wkv_affine_append": [_P, _P, _I64, _I64, _I, _I, _P, _P, _P, _P, _P, _P, _I64, _I64, _P],
    "wkv_affine_fetch": [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _P, _P, _P],
    "wkv_quantize": [_P, _I64, _I, _I, _P, _P, _P],
    "wkv_fp8_quantize": [_P, _I, _I, _I, _I, _P, _P, _P],
    "wkv_fp8_dequantize": [_P, _P, _I, _I, _I, _I, _P, _P],
    "wkv_dequantize": [_P, _P, _I64, _I, _I, _P, _P],
    "wkv_gather_dequantize": [_P, _P, _I64, _P, _I64, _I, _I, _P, _P],
    "wmoe_router_topk": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _F, _P, _P, _P, _P, _P],
    "wmoe_topk_scores": [_P, _P, _I, _I, _I, _I, _F, _F, _P, _P, _P],
    "wmoe_router_topk_static": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _F, _P, _P, _P, _P],
    "wmoe_permute": [_P, _I, _I, _I, _P, _P, _P, _P],
    "wmoe_workspace_size": [_I, _I, _I, _I, _I, _I],
    "wmoe_route_reduce": [_P, _I64, _P, _P, _I, _I, _I, _P, _P, _P],
    "wmoe_mxfp4_experts": [_P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I, _F, _P, _P, _SZ, _P],
    "wmoe_mxfp4_moe_forward": [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I, _F, _I, _P, _P, _P, _SZ, _P],
    "wmoe_mxfp4_moe_layer": [_P, _I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _F, _F, _P, _P, _P, _P, _I, _F, _I, _P, _P, _P,
                             _P, _P, _P, _SZ, _P],
    "wmoe_mxfp4_moe_forward_ep": [_P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _F, _I, _P, _I,
                                  _I, _P, _P, _SZ, _P],
    "wmoe_affine4_experts": [_P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _F, _P, _P, _SZ, _P],
    "wmoe_affine4_moe_forward": [_P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _I, _F, _I, _P, _P, _P,
                                 _SZ, _P],
}
_RESTYPE = {"w_last_error": ctypes.c_char_p, "wmoe_workspace_size": ctypes.c_size_t,
            "wkv_scores_workspace_size": ctypes.c_size_t, "wmx_linear_workspace_size": ctypes.c_size_t}

_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
    """A whallm_b200 entry point returned an error status."""


def lib():
    """Load the shared library (once).  Raises if it was not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(
                        f"{LIB_PATH} is missing: build it with `python -c \"import __graft_entry__ as g; g.build()\"` "
                        "or `python whallm_b200/build.py`")
                h = ctypes.CDLL(LIB_PATH)
                for name, args in SIGNATURES.items():
                    f = getattr(h, name)
                    f.argtypes = args
                    f.restype = _RESTYPE.get(name, ctypes.c_int)
                _lib = h
    return _lib


def last_error() -> str:
    return lib().w_last_error().decode()


def call(name: str, *args):
    """Call an int-returning entry point and raise on a negative status.

    Invalid arguments raise ValueError (as the reference does for bad shapes),
    everything else RuntimeError."""
    rc = getattr(lib(), name)(*args)
    if rc != WM_OK:
        msg = f"{name}: {last_error()} (status {rc})"
        if rc == WM_ERR_INVALID:
            raise ValueError(msg)
        raise NativeError(msg)
    return rc


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def stream_of(t) -> ctypes.c_void_p:
    """The current CUDA stream of the tensor's device."""
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("whallm_b200 ops take CUDA tensors (no CPU fallback)")
        if t is not None and not t.is_contiguous():
            raise ValueError("whallm_b200 ops take contiguous tensors")
