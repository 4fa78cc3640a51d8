"""Quantized number formats on the device: MXFP4 / affine-4 weights, KV rows.

Python mirror of the reference's format helpers; every function runs one
kernel of ``libwhallm_b200.so`` on the tensors' current CUDA stream.

* ``mxfp4_quantize`` -- ``MXFP4.quantizeBF16`` (Sources/DeepSeekRepack/MXFP4.swift:4-40),
  the bytes ``mx.quantize(mode="mxfp4")`` stores.
* ``mxfp4_dequantize`` -- ``dequant_fp4`` (runtime/deepseek_v4_ssd/deepseek_v41/dequant.py:63-66).
* ``affine4_quantize`` / ``affine4_dequantize`` -- ``mx.quantize/dequantize(bits=4)``.
* ``kv_quantize`` / ``kv_dequantize`` / ``kv_gather_dequantize`` -- the packed
  KV row formats (deepseek_v41/packed_cache.py:24-59, fp8_cache.py:109-190).
"""
from __future__ import annotations

import torch

from . import _lib as L

KV_FORMATS = {
    "fp8_f32_b64": L.WKV_FP8_F32_B64,
    "fp8_ue8m0": L.WKV_FP8_UE8M0_B32,
    "fp4_e4m3": L.WKV_FP4_E4M3_B16,
    "fp4_ue8m0": L.WKV_FP4_UE8M0_B32,
    "mxfp8": L.WKV_MXFP8_B32,
    "mxfp4": L.WKV_MXFP4_B32,
}
KV_BLOCK = {0: 64, 1: 32, 2: 16, 3: 32, 4: 32, 5: 32}
KV_BITS = {0: 8, 1: 8, 2: 4, 3: 4, 4: 8, 5: 4}


def _fmt(fmt) -> int:
    if isinstance(fmt, str):
        if fmt not in KV_FORMATS:
            raise ValueError(f"Invalid packed cache format {fmt!r}")
        return KV_FORMATS[fmt]
    return int(fmt)


def mxfp4_quantize(w: torch.Tensor):
    """bf16 [..., rows, cols] -> (packed uint8 [..., rows, cols/2], scales uint8 [..., rows, cols/32])."""
    if w.dtype != torch.bfloat16:
        raise ValueError("MXFP4 source must be bf16")
    L.require_cuda(w)
    cols = w.shape[-1]
    rows = w.numel() // cols if cols else 0
    packed = torch.empty(*w.shape[:-1], cols // 2, dtype=torch.uint8, device=w.device)
    scales = torch.empty(*w.shape[:-1], cols // 32, dtype=torch.uint8, device=w.device)
    L.call("wmxfp4_quantize", L.ptr(w), rows, cols, L.ptr(packed), L.ptr(scales), L.stream_of(w))
    return packed, scales


def mxfp4_dequantize(packed: torch.Tensor, scales: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """(packed [..., rows, cols/2], scales [..., rows, cols/32]) -> dtype [..., rows, cols], bit-exact."""
    L.require_cuda(packed, scales)
    cols = packed.shape[-1] * 2
    rows = packed.numel() // packed.shape[-1] if packed.shape[-1] else 0
    if scales.shape[-1] * 32 != cols or scales.numel() // max(1, scales.shape[-1]) != rows:
        raise ValueError("MXFP4 scales do not match the packed weights")
    out = torch.empty(*packed.shape[:-1], cols, dtype=dtype, device=packed.device)
    kind = {torch.float32: L.WM_OUT_F32, torch.bfloat16: L.WM_OUT_BF16}[dtype]
    L.call("wmxfp4_dequantize", L.ptr(packed), L.ptr(scales), rows, cols, kind, L.ptr(out), L.stream_of(packed))
    return out


def kv_scores(query: torch.Tensor, payload: torch.Tensor, scales: torch.Tensor, fmt, out=None) -> torch.Tensor:
    """MXFP8PoolingCache.quantized_matmul / index_matmul over completed chunks
    (fp8_cache.py:119-159): bf16 [B, Lq, L] = query [B, Lq, D] @ dequant(K)^T,
    K [B, L, D] stored as "mxfp8" (payload u8 [B, L, D]) or "mxfp4" (payload
    u8 [B, L, D/2]) with E8M0 scales u8 [B, L, D/32]."""
    f = _fmt(fmt)
    if f not in (L.WKV_MXFP8_B32, L.WKV_MXFP4_B32):
        raise ValueError("kv_scores takes an mxfp8 or mxfp4 cache")
    if query.dtype != torch.bfloat16 or query.dim() != 3:
        raise ValueError("query must be bf16 [B, Lq, D]")
    B, Lq, D = query.shape
    if scales.dim() != 3 or scales.shape[0] != B or scales.shape[2] != D // 32:
        raise ValueError("scales must be [B, L, D/32]")
    Lc = scales.shape[1]
    want = D if f == L.WKV_MXFP8_B32 else D // 2
    if tuple(payload.shape) != (B, Lc, want) or payload.dtype != torch.uint8:
        raise ValueError(f"payload must be uint8 [B, L, {want}]")
    q = query.contiguous()
    if out is None:
        out = torch.empty((B, Lq, Lc), dtype=torch.bfloat16, device=q.device)
    nbytes = int(L.lib().wkv_scores_workspace_size(B, Lq, D, Lc))
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=q.device)
    L.require_cuda(q, payload, scales, out)
    L.call("wkv_mx_scores", L.ptr(q), B, Lq, D, L.ptr(payload.contiguous()), L.ptr(scales.contiguous()), Lc, f,
           L.ptr(out), L.ptr(ws), ws.numel(), L.stream_of(q))
    return out


def split_e4m3(x: torch.Tensor):
    """bf16 [rows, cols] -> (hi u8, lo u8 [rows, cols], scales u8 [rows, cols/32]):
    the exact two-term e4m3 operand form of the block-scaled expert kernels."""
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise ValueError("split_e4m3 takes a 2-D bf16 tensor")
    x = x.contiguous()
    rows, cols = x.shape
    hi = torch.empty((rows, cols), dtype=torch.uint8, device=x.device)
    lo = torch.empty_like(hi)
    sc = torch.empty((rows, cols // 32), dtype=torch.uint8, device=x.device)
    L.require_cuda(x, hi, lo, sc)
    L.call("wmx_split_e4m3", L.ptr(x), rows, cols, L.ptr(hi), L.ptr(lo), L.ptr(sc), L.stream_of(x))
    return hi, lo, sc


def affine4_quantize(w: torch.Tensor, group: int = 64):
    """bf16 [..., rows, cols] -> (packed uint32 [..., cols/8] as int32 storage, scales bf16, biases bf16)."""
    if w.dtype != torch.bfloat16:
        raise ValueError("affine4 source must be bf16")
    L.require_cuda(w)
    cols = w.shape[-1]
    rows = w.numel() // cols
    packed = torch.empty(*w.shape[:-1], cols // 8, dtype=torch.int32, device=w.device)
    scales = torch.empty(*w.shape[:-1], cols // group, dtype=torch.bfloat16, device=w.device)
    biases = torch.empty_like(scales)
    L.call("waffine4_quantize", L.ptr(w), rows, cols, group, L.ptr(packed), L.ptr(scales), L.ptr(biases),
           L.stream_of(w))
    return packed, scales, biases


def affine4_dequantize(packed, scales, biases, group: int = 64, dtype=torch.bfloat16) -> torch.Tensor:
    L.require_cuda(packed, scales, biases)
    cols = packed.shape[-1] * 8
    rows = packed.numel() // packed.shape[-1]
    out = torch.empty(*packed.shape[:-1], cols, dtype=dtype, device=packed.device)
    kind = {torch.float32: L.WM_OUT_F32, torch.bfloat16: L.WM_OUT_BF16}[dtype]
    L.call("waffine4_dequantize", L.ptr(packed), L.ptr(scales), L.ptr(biases), rows, cols, group, kind, L.ptr(out),
           L.stream_of(packed))
    return out


def kv_shapes(shape, fmt):
    """(payload shape, scales shape, scales dtype) for bf16 rows of `shape`."""
    f = _fmt(fmt)
    D = shape[-1]
    blk = KV_BLOCK[f]
    if D % blk:
        raise ValueError("Invalid packed cache format or width")
    sdt = torch.float32 if f == L.WKV_FP8_F32_B64 else torch.uint8
    return (*shape[:-1], D * KV_BITS[f] // 8), (*shape[:-1], D // blk), sdt


def kv_quantize(x: torch.Tensor, fmt, payload=None, scales=None):
    """bf16 [..., D] -> (payload uint8, scales).  Writes into payload/scales if given."""
    f = _fmt(fmt)
    if x.dtype != torch.bfloat16:
        raise ValueError("KV rows must be bf16")
    L.require_cuda(x)
    pshape, sshape, sdt = kv_shapes(x.shape, f)
    if payload is None:
        payload = torch.empty(pshape, dtype=torch.uint8, device=x.device)
    if scales is None:
        scales = torch.empty(sshape, dtype=sdt, device=x.device)
    if tuple(payload.shape) != tuple(pshape) or tuple(scales.shape) != tuple(sshape) or scales.dtype != sdt:
        raise ValueError("Invalid packed cache array")
    L.require_cuda(payload, scales)
    D = x.shape[-1]
    rows = x.numel() // D
    L.call("wkv_quantize", L.ptr(x), rows, D, f, L.ptr(payload), L.ptr(scales), L.stream_of(x))
    return payload, scales


def kv_dequantize(payload: torch.Tensor, scales: torch.Tensor, fmt, out=None) -> torch.Tensor:
    f = _fmt(fmt)
    L.require_cuda(payload, scales)
    D = payload.shape[-1] * 8 // KV_BITS[f]
    rows = payload.numel() // payload.shape[-1] if payload.shape[-1] else 0
    if out is None:
        out = torch.empty(*payload.shape[:-1], D, dtype=torch.bfloat16, device=payload.device)
    L.call("wkv_dequantize", L.ptr(payload), L.ptr(scales), rows, D, f, L.ptr(out), L.stream_of(payload))
    return out


def kv_gather_dequantize(payload: torch.Tensor, scales: torch.Tensor, rows_idx: torch.Tensor, fmt) -> torch.Tensor:
    """payload [R, D'] / scales [R, nb]; rows_idx int32 [...] (clipped) -> bf16 [..., D]."""
    f = _fmt(fmt)
    L.require_cuda(payload, scales, rows_idx)
    if rows_idx.dtype != torch.int32:
        raise ValueError("row indices must be int32")
    D = payload.shape[-1] * 8 // KV_BITS[f]
    R = payload.numel() // payload.shape[-1]
    out = torch.empty(*rows_idx.shape, D, dtype=torch.bfloat16, device=payload.device)
    L.call("wkv_gather_dequantize", L.ptr(payload), L.ptr(scales), R, L.ptr(rows_idx), rows_idx.numel(), D, f,
           L.ptr(out), L.stream_of(payload))
    return out
