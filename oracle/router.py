"""Router oracle: gate logits, scores, top-k, renormalisation.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Thin ctypes wrapper over ``oracle/c/router_ref.c``, which evaluates the
reference router (``deepseek_v41/moe.py:58-75``, ``qwen4_exp.py:693-699``,
tie rule ``model.py:548-560``) in the fixed float32 order shared with the
device kernel, so routing indices compare exactly.  ``SCORE_SOFTMAX_BF16`` is
the Qwen gate in the reference's dtypes: bf16 logits (a bf16 ``nn.Linear``,
``qwen4_exp.py:683``), ``softmax(precise=True)`` in float32 returned as bf16
(``:693``), top-k on the bf16 probabilities and a bf16 renormalisation
(``:694-697``), shared gate ``bf16(sigmoid(bf16 logit))`` (``:699``).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

SCORE_SOFTMAX, SCORE_SIGMOID, SCORE_SQRTSOFTPLUS, SCORE_NONE, SCORE_SOFTMAX_BF16 = 0, 1, 2, 3, 4
NO_RENORM = -1.0

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        _lib = ctypes.CDLL(path)
        f = _lib.oracle_router
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_float] + [ctypes.c_void_p] * 5
        for name in ("oracle_exp_n", "oracle_softplus_n"):
            g = getattr(_lib, name)
            g.restype = None
            g.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        _lib.oracle_mxfp4_matmul.restype = None
        _lib.oracle_mxfp4_matmul.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                             ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        _lib.oracle_affine4_matmul.restype = None
        _lib.oracle_affine4_matmul.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_void_p]
    return _lib


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def route(x_bf16_bits, wg_bf16_bits, k: int, score_fn: int, *, logit_bias=None, select_bias=None,
          norm_eps: float = NO_RENORM, route_scale: float = 1.0, wg_shared_bits=None):
    """Returns (logits f32 [T,E], idx int32 [T,k], weights f32 [T,k], shared_w f32 [T] or None).

    idx is in selection order: descending key, ties to the lower expert id."""
    x = np.ascontiguousarray(x_bf16_bits, np.uint16)
    w = np.ascontiguousarray(wg_bf16_bits, np.uint16)
    T, H = x.shape
    E = w.shape[0]
    lb = None if logit_bias is None else np.ascontiguousarray(logit_bias, np.float32)
    sb = None if select_bias is None else np.ascontiguousarray(select_bias, np.float32)
    ws = None if wg_shared_bits is None else np.ascontiguousarray(wg_shared_bits, np.uint16)
    logits = np.zeros((T, E), np.float32)
    idx = np.zeros((T, k), np.int32)
    wts = np.zeros((T, k), np.float32)
    shared = np.zeros((T,), np.float32) if ws is not None else None
    rc = lib().oracle_router(_ptr(x), _ptr(w), _ptr(lb), _ptr(sb), T, H, E, k, score_fn,
                             float(norm_eps), float(route_scale), _ptr(ws), _ptr(logits), _ptr(idx),
                             _ptr(wts), _ptr(shared))
    if rc != 0:
        raise ValueError("unsupported router shape")
    return logits, idx, wts, shared


def exp_f32(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oracle_exp_n(_ptr(x), _ptr(y), x.size)
    return y


def softplus_f32(x):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().oracle_softplus_n(_ptr(x), _ptr(y), x.size)
    return y


def stable_topk_indices(scores, count: int):
    """_stable_topk_indices (model.py:548-560): the `count` largest scores,
    ties resolved by position, returned in ascending index order."""
    s = np.asarray(scores)
    order = np.lexsort((np.broadcast_to(np.arange(s.shape[-1]), s.shape), -s), axis=-1)[..., :count]
    return np.sort(order, axis=-1)
