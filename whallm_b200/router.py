"""Router: gate logits, scores, top-k, renormalisation -- on the device.

Mirrors the reference's routers:
  * ``Gate`` -- deepseek_v41/moe.py:46-75 (score_func softmax / sigmoid /
    sqrtsoftplus, selection bias that picks but does not scale, weights
    normalised by ``sum + 1e-20`` and multiplied by ``route_scale``).
  * ``qwen_route`` -- the routing half of SparseMoE.__call__
    (qwen4_exp.py:692-699) in the reference's dtypes: the gate is a bf16
    ``nn.Linear`` (bf16 logits, :683), ``softmax(precise=True)`` computes in
    float32 and returns bf16 probabilities (:693), top-k selects on those
    (:694-695), ``scores / scores.sum()`` is bf16 arithmetic (:696-697), and
    the shared-expert gate is ``sigmoid`` of a bf16 logit in bf16 (:699).
  * ``stable_topk_indices`` -- model.py:548-560 (ties by position).

Ties are resolved towards the lower expert id, and indices come back in
selection order (descending key).  Logits are accumulated in a fixed float32
order so indices are reproducible bit-for-bit.
"""
from __future__ import annotations

import torch

from . import _lib as L

SCORE_FUNCS = {"softmax": L.WM_SCORE_SOFTMAX, "sigmoid": L.WM_SCORE_SIGMOID,
               "sqrtsoftplus": L.WM_SCORE_SQRTSOFTPLUS, "none": L.WM_SCORE_NONE,
               "softmax_bf16": L.WM_SCORE_SOFTMAX_BF16}


def route(x: torch.Tensor, weight: torch.Tensor, top_k: int, score_func: str = "softmax", *,
          logit_bias: torch.Tensor | None = None, select_bias: torch.Tensor | None = None,
          norm_eps: float | None = None, route_scale: float = 1.0, shared_gate: torch.Tensor | None = None,
          logits_out: torch.Tensor | None = None):
    """x bf16 [..., H], weight bf16 [E, H] -> (weights f32 [..., k], indices int32 [..., k], shared_w or None).

    ``norm_eps=None`` disables renormalisation; ``shared_gate`` bf16 [H] (or
    [1, H]) adds ``shared_w = sigmoid(x . shared_gate)``."""
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise ValueError("router inputs must be bf16")
    H = x.shape[-1]
    E = weight.shape[0]
    if weight.shape[-1] != H:
        raise ValueError("gate weight does not match the hidden size")
    xf = x.reshape(-1, H).contiguous()
    T = xf.shape[0]
    dev = x.device
    for b in (logit_bias, select_bias):
        if b is not None and (b.dtype != torch.float32 or b.numel() != E):
            raise ValueError("router biases must be float32 [E]")
    sg = None if shared_gate is None else shared_gate.reshape(-1).contiguous()
    L.require_cuda(xf, weight, logit_bias, select_bias, sg)
    logits = logits_out if logits_out is not None else torch.empty(T, E, dtype=torch.float32, device=dev)
    idx = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    w = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    shared = torch.empty(T, dtype=torch.float32, device=dev) if sg is not None else None
    L.call("wmoe_router_topk", L.ptr(xf), L.ptr(weight), L.ptr(logit_bias), L.ptr(select_bias), L.ptr(sg), T, H, E,
           top_k, SCORE_FUNCS[score_func], -1.0 if norm_eps is None else float(norm_eps), float(route_scale),
           L.ptr(logits), L.ptr(idx), L.ptr(w), L.ptr(shared), L.stream_of(xf))
    lead = x.shape[:-1]
    return (w.reshape(*lead, top_k), idx.reshape(*lead, top_k),
            None if shared is None else shared.reshape(*lead, 1))


def topk_scores(logits: torch.Tensor, top_k: int, score_func: str = "none", *, select_bias=None,
                norm_eps: float | None = None, route_scale: float = 1.0):
    """Score / top-k / renormalise caller logits f32 [..., E]."""
    if logits.dtype != torch.float32:
        raise ValueError("logits must be float32")
    E = logits.shape[-1]
    lf = logits.reshape(-1, E).contiguous()
    T = lf.shape[0]
    L.require_cuda(lf, select_bias)
    idx = torch.empty(T, top_k, dtype=torch.int32, device=lf.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=lf.device)
    L.call("wmoe_topk_scores", L.ptr(lf), L.ptr(select_bias), T, E, top_k, SCORE_FUNCS[score_func],
           -1.0 if norm_eps is None else float(norm_eps), float(route_scale), L.ptr(idx), L.ptr(w), L.stream_of(lf))
    return w.reshape(*logits.shape[:-1], top_k), idx.reshape(*logits.shape[:-1], top_k)


def stable_topk_indices(scores: torch.Tensor, count: int) -> torch.Tensor:
    """_stable_topk_indices (model.py:548-560): the `count` largest scores,
    ties by position, returned in ascending index order (int32)."""
    _, idx = topk_scores(scores.float().contiguous(), count, "none")
    return torch.sort(idx, dim=-1).values


class Gate:
    """deepseek_v41/moe.py:46-75 on the device.

    ``weight`` bf16 [E, H]; ``bias`` float32 [E] is the selection bias.
    ``logit_bias`` (float32 [E], optional) is added to the logits before the
    score function (used by the synthetic skewed-routing workloads)."""

    def __init__(self, weight: torch.Tensor, topk: int, score_func: str = "sqrtsoftplus",
                 bias: torch.Tensor | None = None, norm_topk_prob: bool = True, route_scale: float = 1.5,
                 logit_bias: torch.Tensor | None = None):
        self.weight = weight
        self.topk = topk
        self.score_func = score_func
        self.bias = bias
        self.norm_topk_prob = norm_topk_prob
        self.route_scale = route_scale
        self.logit_bias = logit_bias

    def __call__(self, x: torch.Tensor):
        norm = 1e-20 if (self.norm_topk_prob and self.topk > 1) else None
        w, idx, _ = route(x, self.weight, self.topk, self.score_func, logit_bias=self.logit_bias,
                          select_bias=self.bias, norm_eps=norm, route_scale=self.route_scale)
        return w, idx


def qwen_route(x, gate_weight, top_k: int, norm_topk_prob: bool = True, shared_gate=None, logit_bias=None):
    """Routing half of SparseMoE.__call__ (qwen4_exp.py:692-699): (scores, indices, shared_w).

    bf16 gate semantics (``softmax_bf16``): selection on bf16 probabilities,
    scores and shared_w are bf16 values (returned as float32 tensors)."""
    return route(x, gate_weight, top_k, "softmax_bf16", logit_bias=logit_bias,
                 norm_eps=0.0 if norm_topk_prob else None, route_scale=1.0, shared_gate=shared_gate)
