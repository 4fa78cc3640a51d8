"""CUDA-core MXFP4 weight stream (expert calls of one or two tokens) vs the CPU oracle.

The default expert path sends calls of at most two tokens on Qwen-class
experts (H <= 4096, I <= 1024) to the weight stream (``csrc/moe_stream.cu``)
and everything else to the block-scaled tensor-core kernels;
``WM_EXPERT_PATH`` forces either, and every test here forces the stream
(DeepSeek-class shapes included).  Checked:

* whole layers and un-reduced switch_mlp rows within max-relative error 2e-2
  of the oracle, for row lengths that take 16-byte
  pieces (1024 values and up) and 8-byte pieces (256, 512), with and without
  a shared expert, both gate/up orders;
* a two-token call gives the same bits as its tokens one at a time (the lane
  sums' reduction tree does not depend on how many tokens a pass carries);
* an expert routed more than twice by the same call (passes over its slots),
  an out-of-range expert id (zeros, no access outside the layer), and token
  groups spanning a wide range of magnitudes (the f16 operand with a
  power-of-two scale per 32 values);
* the stream and the tensor-core path agree within the tolerance on the same
  call.
"""
import numpy as np
import pytest
import torch

import whallm_b200 as W
from oracle import moe as M
from whallm_b200 import synthetic as S

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(autouse=True)
def _stream_path(monkeypatch):
    monkeypatch.setenv("WM_EXPERT_PATH", "stream")


def _np(t):
    return t.cpu().numpy()


def _f32(t):
    return t.float().cpu().numpy()


def _oracle(ex, order, limit):
    if isinstance(ex, W.QwenBatchedExperts):
        return M.MXFP4Experts(_np(ex.gate_up), _np(ex.gate_up_scales), _np(ex.down), _np(ex.down_scales), order, limit)
    return M.MXFP4Experts(_np(ex.w13), _np(ex.w13_scales), _np(ex.w2), _np(ex.w2_scales), order, limit)


def _route(T, k, E, seed, dev):
    rng = np.random.default_rng(seed)
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.05, 1.0, (T, k)).astype(np.float32)
    return idx, w, torch.from_numpy(idx).to(dev), torch.from_numpy(w).to(dev)


@pytest.mark.parametrize("T,E,H,I,k", [(1, 16, 1024, 512, 6), (2, 16, 1024, 512, 6), (1, 8, 512, 256, 3),
                                       (2, 12, 2048, 1024, 4), (1, 9, 7168, 2048, 8), (2, 6, 256, 256, 2)])
def test_stream_moe_forward_vs_oracle(dev, T, E, H, I, k):
    ex = S.make_mxfp4_experts(E + 1, H, I, seed=T * 31 + H, device=dev)
    x = S.make_tokens(T, H, T + I, dev)
    ri, rw, idx, w = _route(T, k, E, T + E, dev)
    out = W.experts_forward(x, idx, ex, weights=w, shared_expert=E, swiglu_limit=10.0)
    orc = _oracle(ex, M.UP_GATE, 10.0)
    ref = M.moe_forward(_f32(x), ri, rw, orc, shared_expert=E)
    err = M.max_rel_err(_f32(out), ref)
    assert err < TOL, err
    un = W.experts_forward(x, idx, ex, swiglu_limit=10.0)
    assert M.max_rel_err(_f32(un), M.switch_mlp(_f32(x), ri, orc)) < TOL


def test_stream_qwen_gate_up_order_vs_oracle(dev):
    T, E, H, I, k = 1, 24, 2048, 512, 10
    lay = S.make_layer("qn", dev, seed=11, E=E, H=H, I=I)
    x = S.make_tokens(T, H, 11, dev)
    ri, rw, idx, w = _route(T, k, E, 11, dev)
    out = W.experts_forward(x, idx, lay.experts, weights=w)
    ref = M.moe_forward(_f32(x), ri, rw, _oracle(lay.experts, M.GATE_UP, 0.0))
    assert M.max_rel_err(_f32(out), ref) < TOL


def test_stream_two_tokens_equal_one_at_a_time(dev):
    E, H, I, k = 12, 1024, 512, 4
    ex = S.make_mxfp4_experts(E + 1, H, I, seed=5, device=dev)
    x = S.make_tokens(2, H, 5, dev)
    idx = torch.tensor([[0, 3, 5, 7], [3, 5, 9, 1]], dtype=torch.int32, device=dev)   # experts 3 and 5 shared
    w = torch.tensor([[0.5, 0.25, 0.125, 0.125], [0.3, 0.3, 0.2, 0.2]], device=dev)
    both = W.experts_forward(x, idx, ex, weights=w, shared_expert=E, swiglu_limit=10.0)
    one = torch.cat([W.experts_forward(x[i:i + 1], idx[i:i + 1], ex, weights=w[i:i + 1], shared_expert=E,
                                       swiglu_limit=10.0) for i in range(2)])
    assert torch.equal(both, one)
    un2 = W.experts_forward(x, idx, ex, swiglu_limit=10.0)
    un1 = torch.cat([W.experts_forward(x[i:i + 1], idx[i:i + 1], ex, swiglu_limit=10.0) for i in range(2)])
    assert torch.equal(un2, un1)


def test_stream_expert_routed_many_times(dev):
    # expert 3 takes five slots of a two-token call: three passes over its rows
    E, H, I = 6, 1024, 512
    ex = S.make_mxfp4_experts(E, H, I, seed=8, device=dev)
    x = S.make_tokens(2, H, 8, dev)
    ri = np.array([[3, 3, 3, 1], [3, 1, 3, 0]], dtype=np.int32)
    rw = np.full((2, 4), 0.25, dtype=np.float32)
    out = W.experts_forward(x, torch.from_numpy(ri).to(dev), ex, weights=torch.from_numpy(rw).to(dev),
                            swiglu_limit=10.0)
    ref = M.moe_forward(_f32(x), ri, rw, _oracle(ex, M.UP_GATE, 10.0))
    assert M.max_rel_err(_f32(out), ref) < TOL


def test_stream_invalid_id_gives_zeros(dev):
    E, H, I = 4, 256, 256
    ex = S.make_mxfp4_experts(E, H, I, seed=2, device=dev)
    x = S.make_tokens(2, H, 2, dev)
    idx = torch.tensor([[0, 1, 2], [3, 0, 77]], dtype=torch.int32, device=dev)
    w = torch.full((2, 3), 0.25, device=dev)
    out = W.experts_forward(x, idx, ex, weights=w, swiglu_limit=10.0)
    assert torch.count_nonzero(out) == 0


def test_stream_wide_dynamic_range_tokens(dev):
    # groups whose values span ~2^100, a zero group, and huge values: the per-group
    # power-of-two scale keeps every product within f32 accuracy of the oracle's
    E, H, I, k = 5, 1024, 512, 2
    ex = S.make_mxfp4_experts(E, H, I, seed=4, device=dev)
    rng = np.random.default_rng(4)
    xv = rng.standard_normal((2, H)).astype(np.float32)
    xv[0, :32] *= np.float32(2.0) ** rng.integers(-60, 40, 32).astype(np.float32)
    xv[0, 32:64] = 0.0
    xv[1, 64:96] *= np.float32(1e30)
    x = torch.from_numpy(xv).to(dev).to(torch.bfloat16)
    ri, rw, idx, w = _route(2, k, E, 4, dev)
    out = W.experts_forward(x, idx, ex, weights=w, swiglu_limit=10.0)
    ref = M.moe_forward(_f32(x), ri, rw, _oracle(ex, M.UP_GATE, 10.0))
    assert M.max_rel_err(_f32(out), ref) < TOL


def test_stream_and_tensor_core_paths_agree(dev, monkeypatch):
    E, H, I, k = 16, 2048, 1024, 6
    ex = S.make_mxfp4_experts(E + 1, H, I, seed=9, device=dev)
    x = S.make_tokens(2, H, 9, dev)
    ri, rw, idx, w = _route(2, k, E, 9, dev)
    stream = W.experts_forward(x, idx, ex, weights=w, shared_expert=E, swiglu_limit=10.0)
    monkeypatch.setenv("WM_EXPERT_PATH", "mma")     # (the autouse fixture set "stream")
    mma = W.experts_forward(x, idx, ex, weights=w, shared_expert=E, swiglu_limit=10.0)
    assert M.max_rel_err(_f32(stream), _f32(mma)) < TOL   # (often the same bf16 bits: both are f32-accurate)
    # the stream forced onto a four-token call (the shared expert's four slots: two passes)
    x4 = S.make_tokens(4, H, 10, dev)
    ri4, rw4, idx4, w4 = _route(4, k, E, 10, dev)
    monkeypatch.setenv("WM_EXPERT_PATH", "stream")
    out4 = W.experts_forward(x4, idx4, ex, weights=w4, shared_expert=E, swiglu_limit=10.0)
    ref4 = M.moe_forward(_f32(x4), ri4, rw4, _oracle(ex, M.UP_GATE, 10.0), shared_expert=E)
    assert M.max_rel_err(_f32(out4), ref4) < TOL


@pytest.mark.parametrize("T,H,I,E,k", [(1, 2048, 512, 40, 10), (2, 4096, 1024, 20, 8), (2, 1024, 256, 12, 4),
                                       (1, 256, 256, 6, 3)])
def test_stream_row_split_combine_equals_combine_launch(dev, monkeypatch, T, H, I, E, k):
    # small calls: the down projection splits the output rows over its CTAs, groups the call before its
    # dependency wait and combines its own rows; the same bits as the grouping launch, the row-chunk
    # split by expert and the separate combine launch (WM_FUSE=0), with a shared-expert weight
    ex = S.make_mxfp4_experts(E + 1, H, I, seed=T * 7 + H, device=dev)
    x = S.make_tokens(T, H, T + H, dev)
    ri, rw, idx, w = _route(T, k, E, T + E + H, dev)
    sw = torch.rand(T, 1, device=dev) + 0.25
    fused = W.experts_forward(x, idx, ex, weights=w, shared_expert=E, shared_w=sw, swiglu_limit=10.0)
    monkeypatch.setenv("WM_FUSE", "0")
    sep = W.experts_forward(x, idx, ex, weights=w, shared_expert=E, shared_w=sw, swiglu_limit=10.0)
    assert torch.equal(fused, sep)
    ref = M.moe_forward(_f32(x), ri, rw, _oracle(ex, M.UP_GATE, 10.0), shared_expert=E,
                         shared_weight=_f32(sw).reshape(-1))
    assert M.max_rel_err(_f32(fused), ref) < TOL
