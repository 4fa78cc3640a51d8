"""Parity at the BASELINE configurations' full sizes.

* DeepSeek-class layer (H 7168, I 2048, 256 routed experts + 1 shared, top-8,
  MXFP4, Zipf-skewed router, ClampedSwiGLU 10): the decode sweep B = 1, 4, 16,
  64 -- routing indices and weights bit-exact against the oracle router, every
  output row within 2e-2 (max-relative, bf16 output) of the oracle layer; the
  4096-token prefill -- routing of all 4096 tokens bit-exact, the outputs of a
  seeded sample of 256 tokens within 2e-2.
* Qwen-class layer (H 2048, I 512, 512 routed experts + 1 shared, top-10, bf16
  gate, Zipf 1.1): decode B = 1 and 32 on every row; a 16384-token prefill
  with all routes exact and 256 sampled rows within 2e-2.
* The reference's constant-weight composition check
  (runtime/tests/test_runtime.py:2466-2528): with weights that MXFP4 stores
  exactly, every expert path gives the analytic dequantize-then-matmul result.

The oracle reads each expert's packed weights from the device only when a
routed token needs it, so a 6 GB layer is never copied whole at once.
"""
import numpy as np
import pytest
import torch

import whallm_b200 as W
from oracle import formats as F
from oracle import moe as M
from oracle import router as R
from whallm_b200 import synthetic as S

pytestmark = pytest.mark.gpu
TOL = 2e-2
SAMPLE = 256


def _np(t):
    return t.cpu().numpy()


def _f32(t):
    return t.float().cpu().numpy()


def _bits(t):
    return _np(t.contiguous().view(torch.int16)).view(np.uint16)


class _PerExpert:
    """An [E, ...] device tensor read by the oracle one expert at a time."""

    def __init__(self, t):
        self.t = t

    def __getitem__(self, e):
        return _np(self.t[e])


def _oracle_experts(ex, order, limit):
    if isinstance(ex, W.QwenBatchedExperts):
        ts = (ex.gate_up, ex.gate_up_scales, ex.down, ex.down_scales)
    else:
        ts = (ex.w13, ex.w13_scales, ex.w2, ex.w2_scales)
    return M.MXFP4Experts(*(_PerExpert(t) for t in ts), order, limit)


def _oracle_route(lay, x):
    cfg = lay.cfg
    xb = _bits(x)
    if lay.name == "ds":
        _, idx, w, _ = R.route(xb, _bits(lay.gate_weight), cfg["k"], R.SCORE_SQRTSOFTPLUS,
                               logit_bias=_np(lay.logit_bias), norm_eps=1e-20, route_scale=1.5)
        return idx, w, None
    _, idx, w, sh = R.route(xb, _bits(lay.gate_weight), cfg["k"], R.SCORE_SOFTMAX_BF16,
                            logit_bias=_np(lay.logit_bias), norm_eps=0.0, wg_shared_bits=_bits(lay.shared_gate).reshape(-1))
    return idx, w, sh


def _device_route(lay, x):
    if lay.name == "ds":
        w, idx = lay.layer.gate(x)
        return idx, w, None
    w, idx, sh = W.qwen_route(x, lay.gate_weight, lay.cfg["k"], True, shared_gate=lay.shared_gate,
                              logit_bias=lay.logit_bias)
    return idx, w, sh.reshape(-1)


def _check(lay, x, rows=None):
    """Run the device layer on all of x; routing exact for every token, the
    output rows `rows` (default all) within TOL of the oracle."""
    out = lay.layer(x)
    idx, w, sh = _device_route(lay, x)
    torch.cuda.synchronize()
    ri, rw, rsh = _oracle_route(lay, x)
    np.testing.assert_array_equal(_np(idx), ri)
    np.testing.assert_array_equal(_np(w).view(np.uint32), rw.view(np.uint32))
    if rsh is not None:
        np.testing.assert_array_equal(_np(sh).view(np.uint32), rsh.view(np.uint32))
    sel = np.arange(x.shape[0]) if rows is None else rows
    order = M.UP_GATE if lay.name == "ds" else M.GATE_UP
    ex = _oracle_experts(lay.experts, order, 10.0 if lay.name == "ds" else 0.0)
    ref = M.moe_forward(_f32(x)[sel], ri[sel], rw[sel], ex, shared_expert=lay.cfg["E"],
                        shared_weight=None if rsh is None else rsh[sel])
    err = M.max_rel_err(_f32(out)[sel], ref)
    assert err < TOL, err
    return err


@pytest.fixture(scope="module")
def ds_layer():
    lay = S.make_layer("ds", torch.device("cuda:0"), seed=0)
    yield lay
    del lay
    torch.cuda.empty_cache()


@pytest.fixture(scope="module")
def qn_layer():
    lay = S.make_layer("qn", torch.device("cuda:0"), seed=0)
    yield lay
    del lay
    torch.cuda.empty_cache()


@pytest.mark.parametrize("B", [1, 4, 16, 64])
def test_ds_decode_full_layer_vs_oracle(dev, ds_layer, B):
    x = S.make_tokens(B, ds_layer.cfg["H"], 100, dev)
    _check(ds_layer, x)


def test_ds_prefill_4096_routes_exact_and_sampled_rows(dev, ds_layer):
    x = S.make_tokens(4096, ds_layer.cfg["H"], 4096, dev)
    rows = np.sort(np.random.default_rng(4096).choice(4096, SAMPLE, replace=False))
    _check(ds_layer, x, rows)


@pytest.mark.parametrize("B", [1, 32])
def test_qn_decode_full_layer_vs_oracle(dev, qn_layer, B):
    x = S.make_tokens(B, qn_layer.cfg["H"], 100, dev)
    _check(qn_layer, x)


def test_qn_prefill_16384_routes_exact_and_sampled_rows(dev, qn_layer):
    x = S.make_tokens(16384, qn_layer.cfg["H"], 16384, dev)
    rows = np.sort(np.random.default_rng(16384).choice(16384, SAMPLE, replace=False))
    _check(qn_layer, x, rows)


def _constant_mxfp4(rows, cols, value, dev):
    """An MXFP4 matrix whose every element is `value` (a power of two times an
    e2m1 value, stored exactly), quantized by the library."""
    return W.mxfp4_quantize(torch.full((rows, cols), value, dtype=torch.bfloat16, device=dev))


@pytest.mark.parametrize("path", [None, "mma", "stream", "f16", "simt"])
@pytest.mark.parametrize("T", [1, 2, 40])
def test_constant_weights_give_the_dequantize_then_matmul_result(dev, path, T):
    """test_runtime.py:2466-2528 restated: experts with constant weights that
    MXFP4 represents exactly (0.125 ... 0.5) give exactly x @ W13^T -> SwiGLU
    -> @ W2^T, per token and expert, in the selected order.  H = I = 256 so
    every expert path (block-scaled, CUDA-core weight stream, f16 tensor-core,
    general CUDA-core) can run it;
    the gate rows are 256 * 0.125 = 32, where silu(32) = 32 in float32, so the
    whole chain is exact."""
    import os
    H = I = 256
    vals = ((0.125, 0.25, 0.375), (0.25, 0.375, 0.5))        # (w1 gate, w2 down, w3 up) per expert
    w13, s13, w2, s2 = [], [], [], []
    for g, d, u in vals:
        pu, su = _constant_mxfp4(I, H, u, dev)
        pg, sg = _constant_mxfp4(I, H, g, dev)
        w13.append(torch.cat([pu, pg]))                          # [w3; w1] (expert_layout.py:43-62)
        s13.append(torch.cat([su, sg]))
        p2, q2 = _constant_mxfp4(H, I, d, dev)
        w2.append(p2)
        s2.append(q2)
    ex = W.BatchedExperts(None, None, torch.stack(w2), torch.stack(s2), None, None, torch.stack(w13), torch.stack(s13))
    x = torch.ones((T, H), dtype=torch.bfloat16, device=dev)
    idx = torch.tensor([[1, 0]] * T, dtype=torch.int32, device=dev)
    old = os.environ.get("WM_EXPERT_PATH")
    try:
        if path:
            os.environ["WM_EXPERT_PATH"] = path
        else:
            os.environ.pop("WM_EXPERT_PATH", None)
        out = W.experts_forward(x, idx, ex)
    finally:
        if old is None:
            os.environ.pop("WM_EXPERT_PATH", None)
        else:
            os.environ["WM_EXPERT_PATH"] = old
    exp = []
    for e in (1, 0):
        g, d, u = vals[e]
        gate, up = H * g, H * u
        h = float(F.round_bf16(np.float32(gate / (1.0 + np.exp(-gate)) * up))[0])
        exp.append(np.float32(I * h * d))
    ref = np.broadcast_to(np.array(exp, np.float32)[None, :, None], (T, 2, H))
    np.testing.assert_array_equal(_f32(out), F.round_bf16(ref))
