"""Dense block-scaled linears (MXFP8 / MXFP4 weights) on the tensor cores.

The reference loads native FP8 checkpoint weights with one E8M0 scale per
32 x 32 block, expands the scales to one per (row, 32 columns) and installs
MXFP8 QuantizedLinear layers over them (``_prepare_common_weights`` and
``nn.quantize(..., mode="mxfp8")``, deepseek_v41_ssd.py:232-261, 353-360); a
layer computes ``mx.quantized_matmul(x, w, scales, transpose=True,
group_size=32, bits=8, mode="mxfp8")``.  ``MXFP8Linear`` keeps that call
shape; the product runs through ``wmx_linear`` (the block-scaled kernel with
e4m3 weight rows as the MMA's A operand and the tokens as two exact e4m3
terms).
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import formats as F


def expand_block_scales(block_scales: torch.Tensor, rows: int) -> torch.Tensor:
    """[ceil(rows/32), K/32] per-block scales -> [rows, K/32] per-row scales
    (``mx.repeat(scale, 32, axis=0)[:rows]``, deepseek_v41_ssd.py:255)."""
    if block_scales.dim() != 2 or block_scales.shape[0] != (rows + 31) // 32:
        raise ValueError(f"native FP8 scale shape is {tuple(block_scales.shape)}; expected "
                         f"({(rows + 31) // 32}, K/32)")
    return block_scales.repeat_interleave(32, dim=0)[:rows].contiguous()


def mx_linear(x: torch.Tensor, weight: torch.Tensor, scales: torch.Tensor, fmt="mxfp8", out=None) -> torch.Tensor:
    """y [..., N] bf16 = x [..., K] @ dequant(weight)^T (MXFP8 u8 [N, K] or MXFP4 u8 [N, K/2], E8M0 [N, K/32])."""
    f = F._fmt(fmt)
    if f not in (L.WKV_MXFP8_B32, L.WKV_MXFP4_B32):
        raise ValueError("mx_linear takes mxfp8 or mxfp4 weights")
    if x.dtype != torch.bfloat16:
        raise ValueError("mx_linear input must be bf16")
    K = x.shape[-1]
    N = weight.shape[0]
    want = K if f == L.WKV_MXFP8_B32 else K // 2
    if weight.dtype != torch.uint8 or tuple(weight.shape) != (N, want):
        raise ValueError(f"weight must be uint8 [N, {want}]")
    if scales.dtype != torch.uint8 or tuple(scales.shape) != (N, K // 32):
        raise ValueError("scales must be uint8 [N, K/32]")
    xf = x.reshape(-1, K).contiguous()
    T = xf.shape[0]
    if out is None:
        out = torch.empty((T, N), dtype=torch.bfloat16, device=x.device)
    if T:
        nbytes = int(L.lib().wmx_linear_workspace_size(T, K, N))
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
        L.require_cuda(xf, weight, scales, out)
        L.call("wmx_linear", L.ptr(xf), T, K, L.ptr(weight.contiguous()), L.ptr(scales.contiguous()), N, f,
               L.ptr(out), L.ptr(ws), ws.numel(), L.stream_of(xf))
    return out.reshape(*x.shape[:-1], N)


class MXFP8Linear:
    """An MXFP8 QuantizedLinear: ``weight`` e4m3 bytes [N, K], ``scales`` E8M0
    [N, K/32], optional ``bias`` [N]."""

    def __init__(self, weight: torch.Tensor, scales: torch.Tensor, bias: torch.Tensor | None = None):
        self.weight, self.scales, self.bias = weight, scales, bias

    @classmethod
    def from_native_fp8(cls, weight: torch.Tensor, block_scales: torch.Tensor, bias=None) -> "MXFP8Linear":
        """Native FP8 weight [N, K] (e4m3 bytes) with E8M0 block scales [ceil(N/32), K/32]."""
        if weight.dim() != 2 or weight.shape[1] % 32:
            raise ValueError("native FP8 input dimension is not divisible by 32")
        return cls(weight.contiguous(), expand_block_scales(block_scales, weight.shape[0]), bias)

    @classmethod
    def quantize(cls, w: torch.Tensor, bias=None) -> "MXFP8Linear":
        """bf16 [N, K] -> MXFP8 (``mx.quantize(mode="mxfp8")``)."""
        p, s = F.kv_quantize(w.to(torch.bfloat16), "mxfp8")
        return cls(p, s, bias)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        y = mx_linear(x, self.weight, self.scales, "mxfp8")
        return y if self.bias is None else y + self.bias.to(y.dtype)
