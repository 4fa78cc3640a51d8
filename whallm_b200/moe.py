"""MoE layers: router + routed experts + top-k combine (+ shared expert).

Drop-in mirrors of the reference's MoE call sites:
  * ``streaming_moe(moe, x, input_ids)`` -- ``_streaming_moe`` (model.py:484-499):
    ``gate -> shared -> switch_mlp -> _route_reduce + shared``.
  * ``route_reduce`` -- ``_route_reduce`` (model.py:502-504).
  * ``MoE`` -- DeepSeek-V4.1 ``MoE.__call__`` (deepseek_v41/moe.py:96-112),
    with the shared expert stored as one more MXFP4 expert (index E) so the
    whole layer is one native call (``moe_layer``: router, experts, combine).
  * ``SparseMoE`` -- Qwen ``SparseMoE.__call__`` (qwen4_exp.py:680-704),
    shared expert gated by ``sigmoid(x . w_sg)``.
  * ``moe_layer`` -- ``wmoe_mxfp4_moe_layer``: the router and the MXFP4
    expert call in one library call (the same bits as ``route`` followed by
    ``experts_forward``).
  * ``TinyMoE`` -- the affine-4 tiny configuration (the Qwen-style bf16 gate:
    softmax top-k, renormalised; no shared expert).
"""
from __future__ import annotations

import torch

from . import _lib as L
from . import experts as X
from .router import SCORE_FUNCS, Gate, qwen_route


def route_reduce(routed: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
    """_route_reduce (model.py:502-504): sum_k routed * scores over the
    un-reduced expert rows [..., k, H] (bf16), accumulated in float32 in k order
    on the device (``wmoe_route_reduce``), bf16 result."""
    if routed.dtype != torch.bfloat16:
        raise ValueError("route_reduce takes the bf16 switch_mlp rows")
    k, H = routed.shape[-2], routed.shape[-1]
    y = routed.reshape(-1, H).contiguous()
    T = y.shape[0] // k
    slots = torch.arange(T * k, dtype=torch.int32, device=routed.device).view(T, k)
    w = scores.reshape(T, k).float().contiguous()
    return rows_reduce(y, slots, w).reshape(*routed.shape[:-2], H)


def rows_reduce(y: torch.Tensor, slots: torch.Tensor, weights: torch.Tensor, add: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """out [T, H] bf16 = sum_j weights[t, j] * y[slots[t, j]] (+ add[t]) on the device
    (``wmoe_route_reduce``): y bf16 [R, H], slots int32 [T, k] (negative: skipped),
    weights f32 [T, k], add f32 [T, H] or None."""
    from . import _lib as L
    if y.dtype != torch.bfloat16 or slots.dtype != torch.int32 or weights.dtype != torch.float32:
        raise ValueError("rows_reduce: y bf16, slots int32, weights float32")
    T, k = slots.shape
    H = y.shape[-1]
    if add is not None and (add.dtype != torch.float32 or tuple(add.shape) != (T, H)):
        raise ValueError("rows_reduce: add must be float32 [T, H]")
    L.require_cuda(y, slots, weights, add)
    out = torch.empty((T, H), dtype=torch.bfloat16, device=y.device) if out is None else out
    L.call("wmoe_route_reduce", L.ptr(y), y.shape[0], L.ptr(slots), L.ptr(weights), T, k, H, L.ptr(add), L.ptr(out),
           L.stream_of(y))
    return out


def streaming_moe(moe, x: torch.Tensor, input_ids=None) -> torch.Tensor:
    """_streaming_moe (model.py:484-499) for an object with ``gate``,
    ``shared_experts`` and ``switch_mlp`` attributes.  ``gate(x[, input_ids])``
    returns ``(indices, scores)`` like mlx-lm's MoEGate."""
    if getattr(moe, "sharding_group", None) is not None:
        raise ValueError("use whallm_b200.ep for expert-parallel layers")
    try:
        indices, scores = moe.gate(x, input_ids)
    except TypeError:
        indices, scores = moe.gate(x)
    shared = moe.shared_experts(x)
    routed = moe.switch_mlp(x, indices)
    return route_reduce(routed, scores) + shared


def moe_layer(x: torch.Tensor, gate_weight: torch.Tensor, top_k: int, experts, *, score_func: str = "softmax",
              logit_bias=None, select_bias=None, norm_eps: float | None = None, route_scale: float = 1.0,
              shared_gate=None, has_shared: bool = False, swiglu_limit: float = 0.0, order=None,
              return_route: bool = False):
    """Router + MXFP4 experts + combine in one library call (``wmoe_mxfp4_moe_layer``).

    Arguments as ``route`` (gate ``gate_weight`` bf16 [n_routed, H]) and
    ``experts_forward`` (``experts`` holds the routed experts, then the shared
    one when ``has_shared``; its weight is ``sigmoid(x . shared_gate)`` when a
    shared gate is given, else 1).  Results are the bits of the two separate
    calls.  Returns out [..., H] bf16, and with ``return_route`` also
    (weights, indices, shared_w or None)."""
    if x.dtype != torch.bfloat16 or gate_weight.dtype != torch.bfloat16:
        raise ValueError("layer inputs must be bf16")
    if isinstance(experts, X.Affine4BatchedExperts):
        raise ValueError("moe_layer takes MXFP4 experts")
    H = x.shape[-1]
    n_routed = gate_weight.shape[0]
    xf = x.reshape(-1, H).contiguous()
    T = xf.shape[0]
    dev = x.device
    if isinstance(experts, X.QwenBatchedExperts):
        w13, s13, w2, s2 = experts.gate_up, experts.gate_up_scales, experts.down, experts.down_scales
        order = X.GATE_UP if order is None else order
    else:
        w13, s13, _ = experts.fused()
        w2, s2 = experts.w2, experts.w2_scales
        order = X.UP_GATE if order is None else order
    E, He, I = X._mx_args(w13, s13, w2, s2)
    if He != H or gate_weight.shape[-1] != H:
        raise ValueError("experts or gate do not match the hidden size")
    if E != n_routed + (1 if has_shared else 0):
        raise ValueError("expert count must be routed experts (+1 shared)")
    for b in (logit_bias, select_bias):
        if b is not None and (b.dtype != torch.float32 or b.numel() != n_routed):
            raise ValueError("router biases must be float32 [n_routed]")
    gw = gate_weight.contiguous()
    sg = None if shared_gate is None else shared_gate.reshape(-1).contiguous()
    logits = torch.empty(T, n_routed, dtype=torch.float32, device=dev)
    idx = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    shared_w = torch.empty(T, dtype=torch.float32, device=dev) if sg is not None else None
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    ws = X._WS.get(dev, X.workspace_size(T, top_k, H, I, E, has_shared))
    L.require_cuda(xf, gw, logit_bias, select_bias, sg, w13, s13, w2, s2)
    L.call("wmoe_mxfp4_moe_layer", L.ptr(xf), T, H, I, L.ptr(gw), L.ptr(logit_bias), L.ptr(select_bias), L.ptr(sg),
           n_routed, top_k, SCORE_FUNCS[score_func], -1.0 if norm_eps is None else float(norm_eps), float(route_scale),
           L.ptr(w13), L.ptr(s13), L.ptr(w2), L.ptr(s2), order, float(swiglu_limit), n_routed if has_shared else -1,
           L.ptr(logits), L.ptr(idx), L.ptr(w), L.ptr(shared_w), L.ptr(out), L.ptr(ws), ws.numel(), L.stream_of(xf))
    lead = x.shape[:-1]
    out = out.reshape(*lead, H)
    if not return_route:
        return out
    return out, (w.reshape(*lead, top_k), idx.reshape(*lead, top_k),
                 None if shared_w is None else shared_w.reshape(*lead, 1))


class MoE:
    """DeepSeek-class routed layer: V4.1 Gate semantics, ClampedSwiGLU(limit),
    MXFP4 experts [E+1, ...] whose last expert is the always-on shared expert."""

    def __init__(self, gate: Gate, experts: X.BatchedExperts, swiglu_limit: float = 0.0, has_shared: bool = True):
        self.gate = gate
        self.experts = experts
        self.limit = float(swiglu_limit)
        self.n_routed = gate.weight.shape[0]
        self.has_shared = has_shared
        if X._expert_count(experts) != self.n_routed + (1 if has_shared else 0):
            raise ValueError("expert count must be routed experts (+1 shared)")

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        g = self.gate
        norm = 1e-20 if (g.norm_topk_prob and g.topk > 1) else None
        return moe_layer(x, g.weight, g.topk, self.experts, score_func=g.score_func, logit_bias=g.logit_bias,
                         select_bias=g.bias, norm_eps=norm, route_scale=g.route_scale, has_shared=self.has_shared,
                         swiglu_limit=self.limit)


class SparseMoE:
    """Qwen-class routed layer (qwen4_exp.py:680-704): softmax top-k,
    renormalised, MXFP4 gate_up/down experts [E+1, ...] with the shared
    expert last, scaled by sigmoid(x . shared_expert_gate)."""

    def __init__(self, gate_weight: torch.Tensor, shared_expert_gate: torch.Tensor | None,
                 experts: X.QwenBatchedExperts, top_k: int, norm_topk_prob: bool = True,
                 logit_bias: torch.Tensor | None = None):
        self.gate_weight = gate_weight
        self.shared_expert_gate = shared_expert_gate
        self.experts = experts
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.logit_bias = logit_bias
        self.n_routed = gate_weight.shape[0]

    def __call__(self, value: torch.Tensor) -> torch.Tensor:
        # the gate of qwen_route: bf16 logits and probabilities, plain renormalisation
        has_shared = X._expert_count(self.experts) > self.n_routed
        return moe_layer(value, self.gate_weight, self.top_k, self.experts, score_func="softmax_bf16",
                         logit_bias=self.logit_bias, norm_eps=0.0 if self.norm_topk_prob else None, route_scale=1.0,
                         shared_gate=self.shared_expert_gate, has_shared=has_shared)


class TinyMoE:
    """The tiny affine-4 configuration: bf16 gate, softmax over E (float32, bf16
    result), top-k, renormalised in bf16 (the SparseMoE gate, qwen4_exp.py:692-697);
    no shared expert."""

    def __init__(self, gate_weight: torch.Tensor, experts: X.Affine4BatchedExperts, top_k: int):
        self.gate_weight = gate_weight
        self.experts = experts
        self.top_k = top_k

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        scores, indices, _ = qwen_route(x, self.gate_weight, self.top_k, True)
        return X.experts_forward(x, indices, self.experts, weights=scores)
