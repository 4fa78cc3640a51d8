"""MoE-layer oracle: experts, SwiGLU, top-k weighted combine.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Restates the reference composition:
  * fused gate/up projection and split: DeepSeek ``w13 = [w3(up); w1(gate)]``
    split as ``(up, gate)`` (expert_layout.py:43-60, model.py:415-417);
    Qwen ``gate_up = [gate; up]`` split as ``(gate, up)`` (qwen4_exp.py:608-611).
  * ClampedSwiGLU in float32: up clipped to +-limit, gate capped at +limit,
    ``silu(gate) * up`` (deepseek_v41/moe.py:30-43); limit 0 = plain SwiGLU
    (qwen4_exp.py:611, 634).
  * down projection, then ``sum_k w_k * y_k`` (+ shared expert)
    (model.py:484-504, deepseek_v41/moe.py:105-112, qwen4_exp.py:692-704).
The quantized matmuls dequantize group by group in C (``oracle/c/moe_ref.c``).
The SwiGLU output is rounded to bf16 before the down projection, as a bf16
activation tensor is in the reference.
"""
from __future__ import annotations

import numpy as np

from . import formats as F
from .router import _ptr, lib

UP_GATE = 0   # DeepSeek w13 = [w3; w1] -> (up, gate)
GATE_UP = 1   # Qwen gate_up = [gate; up] -> (gate, up)


def mxfp4_matmul(x_f32, w_u8, s_u8):
    """y = x @ dequant(w)^T (MLX quantized_matmul, transpose=True, mxfp4, group 32)."""
    x = np.ascontiguousarray(x_f32, np.float32)
    w = np.ascontiguousarray(w_u8, np.uint8)
    s = np.ascontiguousarray(s_u8, np.uint8)
    n, K = x.shape
    rows = w.shape[0]
    assert w.shape[1] * 2 == K and s.shape == (rows, K // 32)
    y = np.empty((n, rows), np.float32)
    lib().oracle_mxfp4_matmul(_ptr(x), n, _ptr(w), _ptr(s), rows, K, _ptr(y))
    return y


def affine4_matmul(x_f32, w_u32, scales_bits, biases_bits, group=64):
    x = np.ascontiguousarray(x_f32, np.float32)
    w = np.ascontiguousarray(w_u32, np.uint32)
    sc = np.ascontiguousarray(scales_bits, np.uint16)
    bi = np.ascontiguousarray(biases_bits, np.uint16)
    n, K = x.shape
    rows = w.shape[0]
    y = np.empty((n, rows), np.float32)
    lib().oracle_affine4_matmul(_ptr(x), n, _ptr(w), _ptr(sc), _ptr(bi), group, rows, K, _ptr(y))
    return y


def swiglu(up, gate, limit: float):
    up = np.asarray(up, np.float32)
    gate = np.asarray(gate, np.float32)
    if limit > 0:
        up = np.clip(up, -limit, limit)
        gate = np.minimum(gate, np.float32(limit))
    with np.errstate(over="ignore"):
        silu = gate / (np.float32(1.0) + np.exp(-gate))
    return (silu * up).astype(np.float32)


def split_proj(proj, order: int):
    I = proj.shape[-1] // 2
    a, b = proj[..., :I], proj[..., I:]
    return (a, b) if order == UP_GATE else (b, a)   # returns (up, gate)


class MXFP4Experts:
    """Stacked MXFP4 experts: w13 [E, 2I, H/2], s13 [E, 2I, H/32], w2 [E, H, I/2], s2 [E, H, I/32]."""

    def __init__(self, w13, s13, w2, s2, order=UP_GATE, limit=0.0):
        self.w13, self.s13, self.w2, self.s2 = w13, s13, w2, s2
        self.order, self.limit = order, float(limit)

    def ffn(self, e: int, x_f32):
        up, gate = split_proj(mxfp4_matmul(x_f32, self.w13[e], self.s13[e]), self.order)
        h = F.round_bf16(swiglu(up, gate, self.limit))
        return mxfp4_matmul(h, self.w2[e], self.s2[e])


class Affine4Experts:
    """Stacked affine-4 experts (gate_up fused as [w13 rows], group `group`)."""

    def __init__(self, w13, sc13, bi13, w2, sc2, bi2, order=GATE_UP, limit=0.0, group=64):
        self.w13, self.sc13, self.bi13 = w13, sc13, bi13
        self.w2, self.sc2, self.bi2 = w2, sc2, bi2
        self.order, self.limit, self.group = order, float(limit), group

    def ffn(self, e: int, x_f32):
        proj = affine4_matmul(x_f32, self.w13[e], self.sc13[e], self.bi13[e], self.group)
        up, gate = split_proj(proj, self.order)
        h = F.round_bf16(swiglu(up, gate, self.limit))
        return affine4_matmul(h, self.w2[e], self.sc2[e], self.bi2[e], self.group)


def switch_mlp(x_f32, idx, experts):
    """_StreamingSwitchGLU.__call__ (model.py:283-343): un-reduced [T, k, H], bf16 values."""
    x = np.asarray(x_f32, np.float32)
    T, k = idx.shape
    out = None
    flat = idx.reshape(-1)
    order = np.argsort(flat, kind="stable")
    bounds = np.flatnonzero(np.diff(flat[order])) + 1
    for pos in np.split(order, bounds):
        if len(pos) == 0:
            continue
        e = int(flat[pos[0]])
        y = experts.ffn(e, x[pos // k])
        if out is None:
            out = np.zeros((T * k, y.shape[-1]), np.float32)
        out[pos] = y
    return F.round_bf16(out).reshape(T, k, -1)


def moe_forward(x_f32, idx, weights, experts, shared_expert=None, shared_weight=None):
    """Routed combine plus optional shared expert over bf16 expert outputs (the
    dtype switch_mlp and shared_experts return), float32 accumulation, bf16 result.

    ``shared_expert`` is an expert id of ``experts`` run for every token with
    weight ``shared_weight[t]`` (1.0 when None), following
    deepseek_v41/moe.py:109-111 and qwen4_exp.py:699-704."""
    x = np.asarray(x_f32, np.float32)
    T, k = idx.shape
    out = None
    flat = idx.reshape(-1)
    order = np.argsort(flat, kind="stable")
    bounds = np.flatnonzero(np.diff(flat[order])) + 1
    w = np.asarray(weights, np.float32).reshape(-1)
    for pos in np.split(order, bounds):
        if len(pos) == 0:
            continue
        e = int(flat[pos[0]])
        y = F.round_bf16(experts.ffn(e, x[pos // k]))      # switch_mlp returns bf16 rows
        if out is None:
            out = np.zeros((T, y.shape[-1]), np.float32)
        np.add.at(out, pos // k, y * w[pos][:, None])
    if shared_expert is not None:
        y = F.round_bf16(experts.ffn(int(shared_expert), x))
        sw = np.ones((T,), np.float32) if shared_weight is None else np.asarray(shared_weight, np.float32)
        out = y * sw[:, None] if out is None else out + y * sw[:, None]
    return F.round_bf16(out)


def permute(idx, E: int):
    """_gather_sort semantics: stable sort of the flattened (token, k) assignments
    by expert.  Returns (offsets [E+1], perm [T*k] sorted slot -> flat index,
    inv [T*k] flat index -> sorted slot)."""
    flat = np.asarray(idx, np.int64).reshape(-1)
    perm = np.argsort(flat, kind="stable").astype(np.int32)
    counts = np.bincount(flat, minlength=E)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size, dtype=np.int32)
    return offsets, perm, inv


def max_rel_err(a, b) -> float:
    """max |a - b| / max |b| (the tolerance metric used by the parity tests)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.max(np.abs(b))
    return float(np.max(np.abs(a - b)) / den) if den > 0 else float(np.max(np.abs(a - b)))
