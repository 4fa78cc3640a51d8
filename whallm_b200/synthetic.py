"""Seeded synthetic workloads for the BASELINE configurations.

No checkpoints or datasets are available, so every configuration is built
from seeded random tensors with the reference's shapes and distributions:

  tiny  -- H 1024, I 512, E 16, top-4, no shared expert; gate/up [512x1024]
           and down [1024x512] ~ N(0, 0.02) -> bf16 -> affine-4 (group 64);
           router [16x1024] ~ N(0, 0.02); softmax, top-4, renormalised;
           64 tokens ~ N(0, 1).
  ds    -- H 7168, I 2048, E 256 + 1 shared, top-8, MXFP4 from N(0, 0.02);
           router logits ~ N(0, 1) (gate rows ~ N(0, 1/H)) plus a per-expert
           logit bias ln p_e, p_e ~ 1/rank^1.0 (Zipf) over a seeded
           permutation of ranks; V4.1 Gate scoring (sqrt-softplus, weights
           renormalised with eps 1e-20, route scale 1.5), ClampedSwiGLU(10).
  qn    -- H 2048, I 512, E 512 + 1 shared (I 512), top-10, MXFP4 from
           N(0, 0.02); Zipf 1.1 logit bias; softmax, renormalised; shared
           expert gated by sigmoid(x . w_sg).
  kv    -- 576-wide bf16 rows (512 latent + 64 rope) ~ N(0, 1).

Expert weights are generated and quantized on the device, one expert at a
time, with the library's own MXFP4 / affine-4 quantizers.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import experts as X
from . import formats as F
from .moe import MoE, SparseMoE, TinyMoE
from .router import Gate

CONFIGS = {
    "tiny": dict(H=1024, I=512, E=16, k=4, shared=False, fmt="affine4", zipf=None, tokens=64),
    "ds": dict(H=7168, I=2048, E=256, k=8, shared=True, fmt="mxfp4", zipf=1.0, tokens=16),
    "qn": dict(H=2048, I=512, E=512, k=10, shared=True, fmt="mxfp4", zipf=1.1, tokens=32),
}


def zipf_logit_bias(E: int, alpha: float, seed: int) -> torch.Tensor:
    """b_e = ln p_e, p_e proportional to 1/rank_e^alpha, ranks a seeded permutation of 1..E (float32, CPU)."""
    g = torch.Generator().manual_seed(seed)
    rank = torch.randperm(E, generator=g).double() + 1.0
    p = rank.pow(-alpha)
    p = p / p.sum()
    return p.log().float()


def _normal(shape, std, gen, device):
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).mul_(std)


def make_mxfp4_experts(E: int, H: int, I: int, seed: int, device, qwen: bool = False, std: float = 0.02):
    """E experts, weights ~ N(0, std) fp32 -> bf16 -> MXFP4 on the device."""
    w13 = torch.empty(E, 2 * I, H // 2, dtype=torch.uint8, device=device)
    s13 = torch.empty(E, 2 * I, H // 32, dtype=torch.uint8, device=device)
    w2 = torch.empty(E, H, I // 2, dtype=torch.uint8, device=device)
    s2 = torch.empty(E, H, I // 32, dtype=torch.uint8, device=device)
    gen = torch.Generator(device=device).manual_seed(seed)
    for e in range(E):
        a = _normal((2 * I, H), std, gen, device).to(torch.bfloat16)
        p, s = F.mxfp4_quantize(a)
        w13[e].copy_(p)
        s13[e].copy_(s)
        b = _normal((H, I), std, gen, device).to(torch.bfloat16)
        p, s = F.mxfp4_quantize(b)
        w2[e].copy_(p)
        s2[e].copy_(s)
    if qwen:
        return X.QwenBatchedExperts(w13, s13, w2, s2)
    return X.BatchedExperts(None, None, w2, s2, None, None, w13, s13)


def make_affine4_experts(E: int, H: int, I: int, seed: int, device, group: int = 64, std: float = 0.02):
    w13 = torch.empty(E, 2 * I, H // 8, dtype=torch.int32, device=device)
    sc13 = torch.empty(E, 2 * I, H // group, dtype=torch.bfloat16, device=device)
    bi13 = torch.empty_like(sc13)
    w2 = torch.empty(E, H, I // 8, dtype=torch.int32, device=device)
    sc2 = torch.empty(E, H, I // group, dtype=torch.bfloat16, device=device)
    bi2 = torch.empty_like(sc2)
    gen = torch.Generator(device=device).manual_seed(seed)
    for e in range(E):
        a = _normal((2 * I, H), std, gen, device).to(torch.bfloat16)
        p, s, b = F.affine4_quantize(a, group)
        w13[e].copy_(p); sc13[e].copy_(s); bi13[e].copy_(b)
        c = _normal((H, I), std, gen, device).to(torch.bfloat16)
        p, s, b = F.affine4_quantize(c, group)
        w2[e].copy_(p); sc2[e].copy_(s); bi2[e].copy_(b)
    return X.Affine4BatchedExperts(w13, sc13, bi13, w2, sc2, bi2, group, X.GATE_UP)


@dataclass
class Layer:
    name: str
    cfg: dict
    layer: object          # MoE / SparseMoE / TinyMoE
    gate_weight: torch.Tensor
    logit_bias: torch.Tensor | None
    shared_gate: torch.Tensor | None
    experts: object


def make_layer(name: str, device, seed: int = 0, E: int | None = None, H: int | None = None,
               I: int | None = None) -> Layer:
    """Build one synthetic layer (shape overrides are for small test cases)."""
    cfg = dict(CONFIGS[name])
    if E is not None:
        cfg["E"] = E
    if H is not None:
        cfg["H"] = H
    if I is not None:
        cfg["I"] = I
    H_, I_, E_, k = cfg["H"], cfg["I"], cfg["E"], cfg["k"]
    gen = torch.Generator(device=device).manual_seed(seed + 1)
    if name == "tiny":
        gw = _normal((E_, H_), 0.02, gen, device).to(torch.bfloat16)
        ex = make_affine4_experts(E_, H_, I_, seed + 2, device)
        return Layer(name, cfg, TinyMoE(gw, ex, k), gw, None, None, ex)
    gw = _normal((E_, H_), 1.0 / math.sqrt(H_), gen, device).to(torch.bfloat16)
    lb = zipf_logit_bias(E_, cfg["zipf"], seed + 3).to(device)
    n_exp = E_ + (1 if cfg["shared"] else 0)
    if name == "ds":
        ex = make_mxfp4_experts(n_exp, H_, I_, seed + 2, device)
        gate = Gate(gw, k, "sqrtsoftplus", bias=None, norm_topk_prob=True, route_scale=1.5, logit_bias=lb)
        return Layer(name, cfg, MoE(gate, ex, swiglu_limit=10.0, has_shared=cfg["shared"]), gw, lb, None, ex)
    ex = make_mxfp4_experts(n_exp, H_, I_, seed + 2, device, qwen=True)
    sg = _normal((1, H_), 1.0 / math.sqrt(H_), gen, device).to(torch.bfloat16)
    return Layer(name, cfg, SparseMoE(gw, sg, ex, k, True, logit_bias=lb), gw, lb, sg, ex)


def make_tokens(T: int, H: int, seed: int, device) -> torch.Tensor:
    gen = torch.Generator(device=device).manual_seed(seed + 7)
    return torch.randn((T, H), generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
