"""The tcgen05 expert path (MXFP4, H and I multiples of 128) vs the oracle and
vs the CUDA-core GEMV path.

* prefill-shaped routing: hundreds of tokens per expert, so every expert
  spans several 128-token tiles;
* DeepSeek-class full width (H 7168, I 2048) with hot experts;
* the two device paths agree to within the bf16 output tolerance.
"""
import os

import numpy as np
import pytest
import torch

import whallm_b200 as W
from oracle import moe as M
from whallm_b200 import synthetic as S

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _f32(t):
    return t.float().cpu().numpy()


def _oracle(lay, order, limit):
    ex = lay.experts
    if isinstance(ex, W.QwenBatchedExperts):
        return M.MXFP4Experts(ex.gate_up.cpu().numpy(), ex.gate_up_scales.cpu().numpy(), ex.down.cpu().numpy(),
                              ex.down_scales.cpu().numpy(), order, limit)
    return M.MXFP4Experts(ex.w13.cpu().numpy(), ex.w13_scales.cpu().numpy(), ex.w2.cpu().numpy(),
                          ex.w2_scales.cpu().numpy(), order, limit)


def _simt(fn):
    old = os.environ.get("WM_EXPERT_PATH")
    os.environ["WM_EXPERT_PATH"] = "simt"
    try:
        return fn()
    finally:
        if old is None:
            del os.environ["WM_EXPERT_PATH"]
        else:
            os.environ["WM_EXPERT_PATH"] = old


@pytest.mark.parametrize("T,E,H,I", [(300, 8, 1024, 256), (700, 4, 512, 512), (64, 4, 7168, 2048), (40, 6, 2048, 512)])
def test_tc_many_tokens_per_expert_vs_oracle(dev, T, E, H, I):
    lay = S.make_layer("ds", dev, seed=T + H, E=E, H=H, I=I)
    x = S.make_tokens(T, H, T, dev)
    k = min(lay.cfg["k"], E)
    w, idx, _ = W.route(x, lay.gate_weight, k, "sqrtsoftplus", logit_bias=lay.logit_bias, norm_eps=1e-20,
                        route_scale=1.5)
    out = W.experts_forward(x, idx, lay.experts, weights=w, shared_expert=E, swiglu_limit=10.0)
    ref = M.moe_forward(_f32(x), idx.cpu().numpy(), w.cpu().numpy(), _oracle(lay, M.UP_GATE, 10.0), shared_expert=E)
    err = M.max_rel_err(_f32(out), ref)
    assert err < TOL, err
    un = W.experts_forward(x, idx, lay.experts, swiglu_limit=10.0)
    ref_un = M.switch_mlp(_f32(x), idx.cpu().numpy(), _oracle(lay, M.UP_GATE, 10.0))
    assert M.max_rel_err(_f32(un), ref_un) < TOL


@pytest.mark.parametrize("name,T", [("ds", 16), ("qn", 40), ("ds", 257)])
def test_tc_agrees_with_cuda_core_path(dev, name, T):
    E = 32 if name == "ds" else 64
    lay = S.make_layer(name, dev, seed=11, E=E, H=1024 if name == "ds" else 2048, I=512)
    x = S.make_tokens(T, lay.cfg["H"], 11, dev)
    a = lay.layer(x)
    b = _simt(lambda: lay.layer(x))
    assert M.max_rel_err(_f32(a), _f32(b)) < TOL


def test_tc_qwen_gate_up_order_vs_oracle(dev):
    T, E, H, I, k = 96, 16, 2048, 512, 10
    lay = S.make_layer("qn", dev, seed=5, E=E, H=H, I=I)
    x = S.make_tokens(T, H, 5, dev)
    scores, idx, sw = W.qwen_route(x, lay.gate_weight, k, True, shared_gate=lay.shared_gate, logit_bias=lay.logit_bias)
    out = W.experts_forward(x, idx, lay.experts, weights=scores, shared_expert=E, shared_w=sw)
    ref = M.moe_forward(_f32(x), idx.cpu().numpy(), scores.cpu().numpy(), _oracle(lay, M.GATE_UP, 0.0),
                        shared_expert=E, shared_weight=sw.reshape(-1).cpu().numpy())
    assert M.max_rel_err(_f32(out), ref) < TOL
