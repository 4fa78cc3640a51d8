"""The block-scaled tcgen05 expert path (MXFP4 weights straight into
kind::mxf8f6f4 MMAs, tokens as two exact e4m3 terms) on the device.

* the two-term split kernel is bit-exact against the oracle restatement;
* DeepSeek- and Qwen-shaped layers through the default (block-scaled) path
  match the oracle within the north-star tolerance (2e-2 max-relative, bf16
  output) in the decode (32-token tiles) and prefill (128-token tiles)
  configurations, and agree with the f16 tensor-core path and the CUDA-core
  path on the same inputs.
"""
import os

import numpy as np
import pytest
import torch

import whallm_b200 as W
from oracle import formats as F
from oracle import moe as M
from whallm_b200 import synthetic as S

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _with_path(path, fn):
    old = os.environ.get("WM_EXPERT_PATH")
    if path is None:
        os.environ.pop("WM_EXPERT_PATH", None)
    else:
        os.environ["WM_EXPERT_PATH"] = path
    try:
        return fn()
    finally:
        if old is None:
            os.environ.pop("WM_EXPERT_PATH", None)
        else:
            os.environ["WM_EXPERT_PATH"] = old


@pytest.mark.parametrize("rows,cols", [(1, 32), (37, 7168), (300, 2048)])
def test_split_bitexact_vs_oracle(dev, rows, cols):
    g = torch.Generator(device=dev).manual_seed(rows + cols)
    x = torch.randn((rows, cols), generator=g, device=dev)
    x[0, :32] *= torch.logspace(-8, 8, 32, device=dev)
    if rows > 2:
        x[1, :32] = 0.0
        x[2] *= 1e-30
    xb = x.to(torch.bfloat16)
    hi, lo, sc = W.split_e4m3(xb)
    rh, rl, rs = F.split_e4m3(xb.view(torch.int16).cpu().numpy().view(np.uint16))
    np.testing.assert_array_equal(hi.cpu().numpy(), rh)
    np.testing.assert_array_equal(lo.cpu().numpy(), rl)
    np.testing.assert_array_equal(sc.cpu().numpy(), rs)


def _oracle_layer(lay, x):
    ex = lay.experts
    if isinstance(ex, W.QwenBatchedExperts):
        o = M.MXFP4Experts(*(t.cpu().numpy() for t in (ex.gate_up, ex.gate_up_scales, ex.down, ex.down_scales)),
                           M.GATE_UP, 0.0)
        w, idx, sw = W.qwen_route(x, lay.gate_weight, lay.cfg["k"], True, shared_gate=lay.shared_gate,
                                  logit_bias=lay.logit_bias)
        return M.moe_forward(x.float().cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), o,
                             shared_expert=lay.cfg["E"], shared_weight=sw.reshape(-1).cpu().numpy())
    o = M.MXFP4Experts(*(t.cpu().numpy() for t in (ex.w13, ex.w13_scales, ex.w2, ex.w2_scales)), M.UP_GATE, 10.0)
    w, idx = lay.layer.gate(x)
    return M.moe_forward(x.float().cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), o, shared_expert=lay.cfg["E"])


@pytest.mark.parametrize("name,T,E,H,I", [("ds", 1, 16, 7168, 2048), ("ds", 16, 16, 7168, 2048),
                                          ("ds", 64, 32, 1024, 512), ("ds", 200, 8, 1024, 256),
                                          ("qn", 32, 64, 2048, 512), ("qn", 130, 16, 2048, 512)])
def test_block_scaled_layer_vs_oracle(dev, name, T, E, H, I):
    lay = S.make_layer(name, dev, seed=T + E, E=E, H=H, I=I)
    x = S.make_tokens(T, H, T, dev)
    out = _with_path(None, lambda: lay.layer(x))
    ref = _oracle_layer(lay, x)
    err = M.max_rel_err(out.float().cpu().numpy(), ref)
    assert err < TOL, err


@pytest.mark.parametrize("T,I", [(4, 512), (64, 512), (300, 512), (9, 256)])
def test_block_scaled_agrees_with_f16_and_cuda_core_paths(dev, T, I):
    # I = 256: the CUDA-core down projection has 8 scale groups per row, each split over 4 lanes
    lay = S.make_layer("ds", dev, seed=7, E=16, H=1024, I=I)
    x = S.make_tokens(T, 1024, 3, dev)
    a = _with_path(None, lambda: lay.layer(x)).float().cpu().numpy()
    b = _with_path("f16", lambda: lay.layer(x)).float().cpu().numpy()
    c = _with_path("simt", lambda: lay.layer(x)).float().cpu().numpy()
    assert M.max_rel_err(a, b) < TOL
    assert M.max_rel_err(a, c) < TOL


def test_block_scaled_unreduced_switch_mlp(dev):
    lay = S.make_layer("ds", dev, seed=9, E=8, H=1024, I=256)
    x = S.make_tokens(5, 1024, 9, dev)
    w, idx = lay.layer.gate(x)
    un = W.experts_forward(x, idx, lay.experts, swiglu_limit=10.0)
    o = M.MXFP4Experts(*(t.cpu().numpy() for t in (lay.experts.w13, lay.experts.w13_scales, lay.experts.w2,
                                                      lay.experts.w2_scales)), M.UP_GATE, 10.0)
    ref = M.switch_mlp(x.float().cpu().numpy(), idx.cpu().numpy(), o)
    assert M.max_rel_err(un.float().cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("T,E,H,I,k", [(512, 8, 1024, 512, 4), (300, 6, 2048, 1024, 3), (1024, 16, 1024, 256, 8)])
def test_prefill_cta_pair_vs_single_cta_and_oracle(dev, monkeypatch, T, E, H, I, k):
    # prefill-size calls (more than 32 tokens per expert) on the cta_group::2 configuration
    # (WM_MX_PAIR=1: two CTAs per 256-row MMA, each staging one token term) against the single-CTA
    # configuration and the oracle, with the shared expert and un-reduced rows
    import numpy as np
    from oracle import moe as M
    ex = S.make_mxfp4_experts(E + 1, H, I, seed=T + I, device=dev)
    x = S.make_tokens(T, H, T, dev)
    rng = np.random.default_rng(T)
    ri = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    rw = rng.uniform(0.05, 1.0, (T, k)).astype(np.float32)
    idx, w = torch.from_numpy(ri).to(dev), torch.from_numpy(rw).to(dev)
    monkeypatch.delenv("WM_MX_PAIR", raising=False)
    single = W.experts_forward(x, idx, ex, weights=w, shared_expert=E, swiglu_limit=10.0)
    monkeypatch.setenv("WM_MX_PAIR", "1")
    pair = W.experts_forward(x, idx, ex, weights=w, shared_expert=E, swiglu_limit=10.0)
    pair_un = W.experts_forward(x, idx, ex, swiglu_limit=10.0)
    orc = M.MXFP4Experts(ex.w13.cpu().numpy(), ex.w13_scales.cpu().numpy(), ex.w2.cpu().numpy(),
                         ex.w2_scales.cpu().numpy(), M.UP_GATE, 10.0)
    xf = x.float().cpu().numpy()
    ref = M.moe_forward(xf, ri, rw, orc, shared_expert=E)
    assert M.max_rel_err(pair.float().cpu().numpy(), ref) < 2e-2
    assert M.max_rel_err(single.float().cpu().numpy(), ref) < 2e-2
    assert M.max_rel_err(pair.float().cpu().numpy(), single.float().cpu().numpy()) < 2e-2
    assert M.max_rel_err(pair_un.float().cpu().numpy(), M.switch_mlp(xf, ri, orc)) < 2e-2
