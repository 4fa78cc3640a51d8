"""One-call routed-expert layer (``wmoe_mxfp4_moe_layer`` / ``moe_layer``) vs the
router and the expert call run separately.

Logits, indices, weights, the shared gate and the layer output must be the
separate calls' bits, on the CUDA-core weight stream (Qwen-class one- and
two-token calls) and the block-scaled path, for every score function, with
and without selection and logit biases, for expert counts on both of the
router's top-k kernels (at most 128 experts: one warp per token; more: one
CTA per token), and the output within the north-star tolerance of the CPU
oracle.
"""
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


def _np(t):
    return t.cpu().numpy()


def _gate(n_routed, H, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return (torch.randn(n_routed, H, generator=g, device=dev) / H ** 0.5).to(torch.bfloat16)


def _separate(x, gw, k, ex, score, lb, sb, eps, scale, sg, has_shared, limit):
    n_routed = gw.shape[0]
    w, idx, sw = W.route(x, gw, k, score, logit_bias=lb, select_bias=sb, norm_eps=eps, route_scale=scale,
                         shared_gate=sg)
    out = W.experts_forward(x, idx, ex, weights=w, shared_expert=n_routed if has_shared else -1, shared_w=sw,
                            swiglu_limit=limit)
    return out, w, idx, sw


def _check(dev, T, H, I, n_routed, k, score, *, has_shared=True, qwen=False, lb=False, sb=False, eps=None,
           scale=1.0, shared_gate=False, limit=0.0, path=None, monkeypatch=None, oracle=True):
    if path is not None:
        monkeypatch.setenv("WM_EXPERT_PATH", path)
    E = n_routed + (1 if has_shared else 0)
    ex = S.make_mxfp4_experts(E, H, I, seed=T + H + n_routed, device=dev, qwen=qwen)
    gw = _gate(n_routed, H, n_routed + k, dev)
    x = S.make_tokens(T, H, T * 3 + k, dev)
    rng = np.random.default_rng(n_routed * 7 + T)
    lbt = torch.from_numpy(rng.normal(0, 1, n_routed).astype(np.float32)).to(dev) if lb else None
    sbt = torch.from_numpy(rng.normal(0, 0.1, n_routed).astype(np.float32)).to(dev) if sb else None
    sg = _gate(1, H, 99, dev) if shared_gate else None
    ref_out, ref_w, ref_idx, ref_sw = _separate(x, gw, k, ex, score, lbt, sbt, eps, scale, sg, has_shared, limit)
    out, (w, idx, sw) = W.moe_layer(x, gw, k, ex, score_func=score, logit_bias=lbt, select_bias=sbt, norm_eps=eps,
                                    route_scale=scale, shared_gate=sg, has_shared=has_shared, swiglu_limit=limit,
                                    return_route=True)
    assert torch.equal(idx, ref_idx)
    assert torch.equal(w.view(torch.int32), ref_w.view(torch.int32))
    if sg is not None:
        assert torch.equal(sw.reshape(-1).view(torch.int32), ref_sw.reshape(-1).view(torch.int32))
    assert torch.equal(out, ref_out)
    again = W.moe_layer(x, gw, k, ex, score_func=score, logit_bias=lbt, select_bias=sbt, norm_eps=eps,
                        route_scale=scale, shared_gate=sg, has_shared=has_shared, swiglu_limit=limit)
    assert torch.equal(again, out)
    if oracle:
        if isinstance(ex, W.QwenBatchedExperts):
            orc = M.MXFP4Experts(_np(ex.gate_up), _np(ex.gate_up_scales), _np(ex.down), _np(ex.down_scales),
                                 M.GATE_UP, limit)
        else:
            orc = M.MXFP4Experts(_np(ex.w13), _np(ex.w13_scales), _np(ex.w2), _np(ex.w2_scales), M.UP_GATE, limit)
        ref = M.moe_forward(_f32(x), _np(idx), _np(w), orc, shared_expert=n_routed if has_shared else None,
                            shared_weight=None if sw is None else _f32(sw).reshape(-1))
        assert M.max_rel_err(_f32(out), ref) < TOL


@pytest.mark.parametrize("T", [1, 2])
def test_qwen_class_layer_on_the_weight_stream(dev, T):
    # the Qwen gate (bf16 logits and probabilities), shared gate, logit bias; the weight stream
    _check(dev, T, 2048, 512, 512, 10, "softmax_bf16", qwen=True, lb=True, eps=0.0, shared_gate=True)


@pytest.mark.parametrize("T", [1, 2])
def test_deepseek_class_layer_on_the_block_scaled_path(dev, T):
    # V4.1 gate (sqrt-softplus, selection bias, eps 1e-20, scale 1.5), ClampedSwiGLU; block-scaled path
    _check(dev, T, 7168, 2048, 64, 8, "sqrtsoftplus", sb=True, lb=True, eps=1e-20, scale=1.5, limit=10.0)


@pytest.mark.parametrize("score", ["softmax", "sigmoid", "sqrtsoftplus", "none", "softmax_bf16"])
@pytest.mark.parametrize("n_routed", [40, 200])
def test_every_score_function_on_both_top_k_kernels(dev, score, n_routed):
    # 40 experts: the separate router takes one warp per token; 200: one CTA per token
    eps = None if score == "none" else 1e-20
    _check(dev, 1, 1024, 512, n_routed, 6, score, sb=True, eps=eps, scale=1.5, shared_gate=score == "softmax_bf16",
           limit=10.0, oracle=False)


@pytest.mark.parametrize("path", ["mma", "stream"])
def test_forced_paths_and_no_shared_expert(dev, monkeypatch, path):
    _check(dev, 2, 1024, 512, 96, 4, "softmax", has_shared=False, eps=0.0, path=path, monkeypatch=monkeypatch)


@pytest.mark.parametrize("T", [4, 40])
def test_larger_calls(dev, T):
    _check(dev, T, 2048, 512, 128, 8, "softmax_bf16", qwen=True, lb=True, eps=0.0, shared_gate=True)
