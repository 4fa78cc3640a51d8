"""Device permute and expert forward vs the CPU oracle.

* permute: offsets / perm / inv identical to a stable argsort (bit-exact),
  invalid ids flagged (offsets[E] = -1) with no out-of-range access.
* experts: un-reduced switch_mlp output and the fused moe_forward (top-k
  combine + shared expert) within max-relative error 2e-2 of the oracle
  (bf16 output), for DeepSeek (w13 = [up; gate],
  ClampedSwiGLU 10), Qwen (gate_up = [gate; up], sigmoid-gated shared) and the
  affine-4 tiny configuration.
* grouping invariance: a batch gives bit-identical rows to the same tokens run
  one at a time on the same expert path (test_qwen_grouped_experts.py:23-45
  asks the same of MLX).
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


def _np(t):
    return t.cpu().numpy()


def _f32(t):
    return t.float().cpu().numpy()


def _mx_oracle(ex, order, limit):
    if isinstance(ex, W.QwenBatchedExperts):
        return M.MXFP4Experts(_np(ex.gate_up), _np(ex.gate_up_scales), _np(ex.down), _np(ex.down_scales), order, limit)
    return M.MXFP4Experts(_np(ex.w13), _np(ex.w13_scales), _np(ex.w2), _np(ex.w2_scales), order, limit)


@pytest.mark.parametrize("T,k,E", [(1, 8, 256), (64, 9, 257), (4096, 8, 256), (300, 10, 513), (7, 3, 5)])
def test_permute_matches_stable_argsort(dev, T, k, E):
    rng = np.random.default_rng(T + k + E)
    p = rng.zipf(1.3, (T, k)) % E
    idx = torch.from_numpy(p.astype(np.int32)).to(dev)
    off, perm, inv = W.permute(idx, E)
    r_off, r_perm, r_inv = M.permute(p, E)
    np.testing.assert_array_equal(_np(off), r_off)
    np.testing.assert_array_equal(_np(perm), r_perm)
    np.testing.assert_array_equal(_np(inv), r_inv)


def test_permute_flags_out_of_range_ids(dev):
    idx = torch.tensor([[0, 3], [9, 1]], dtype=torch.int32, device=dev)
    off, _, _ = W.permute(idx, 4)
    assert _np(off)[-1] == -1


def test_moe_forward_invalid_id_gives_zeros(dev):
    lay = S.make_layer("ds", dev, seed=5, E=4, H=256, I=64)
    x = S.make_tokens(3, 256, 5, dev)
    idx = torch.tensor([[0, 1, 2, 3, 0, 1, 2, 3], [0, 1, 2, 3, 0, 1, 2, 77], [0] * 8], dtype=torch.int32, device=dev)
    w = torch.full((3, 8), 0.125, device=dev)
    out = W.experts_forward(x, idx, lay.experts, weights=w, swiglu_limit=10.0)
    assert torch.count_nonzero(out) == 0


def _ds_case(dev, T, E, H, I, seed):
    lay = S.make_layer("ds", dev, seed=seed, E=E, H=H, I=I)
    x = S.make_tokens(T, H, seed, dev)
    return lay, x


@pytest.mark.parametrize("T,E,H,I", [(1, 16, 7168, 2048), (16, 16, 7168, 2048), (5, 8, 1024, 256), (33, 12, 512, 512)])
def test_ds_moe_forward_vs_oracle(dev, T, E, H, I):
    lay, x = _ds_case(dev, T, E, H, I, seed=T + E)
    gate = lay.layer.gate
    wts, idx = gate(x)
    out = lay.layer(x)
    xo = _f32(x)
    lg, ri, rw, _ = R.route(F.f32_to_bf16_bits(xo), _np(lay.gate_weight.view(torch.int16)).view(np.uint16), gate.topk,
                            R.SCORE_SQRTSOFTPLUS, logit_bias=_np(lay.logit_bias), norm_eps=1e-20, route_scale=1.5)
    np.testing.assert_array_equal(_np(idx), ri)
    np.testing.assert_array_equal(_np(wts).view(np.uint32), rw.view(np.uint32))
    ex = _mx_oracle(lay.experts, M.UP_GATE, 10.0)
    ref = M.moe_forward(xo, ri, rw, ex, shared_expert=E)
    err = M.max_rel_err(_f32(out), ref)
    assert err < TOL, err
    # un-reduced switch_mlp output
    store = W.ResidentExpertStore({0: lay.experts})
    sw = W.StreamingSwitchGLU(0, store, W.ClampedSwiGLU(10.0))
    un = sw(x, idx)
    assert un.shape == (T, gate.topk, H)
    ref_un = M.switch_mlp(xo, ri, ex)
    assert M.max_rel_err(_f32(un), ref_un) < TOL
    assert store.metrics.gather_qmm_calls == 2


def test_qwen_sparse_moe_vs_oracle(dev):
    T, E, H, I, k = 24, 64, 2048, 512, 10
    lay = S.make_layer("qn", dev, seed=3, E=E, H=H, I=I)
    x = S.make_tokens(T, H, 3, dev)
    out = lay.layer(x)
    xb = F.f32_to_bf16_bits(_f32(x))
    _, ri, rw, rsh = R.route(xb, _np(lay.gate_weight.view(torch.int16)).view(np.uint16), k, R.SCORE_SOFTMAX_BF16,
                             logit_bias=_np(lay.logit_bias), norm_eps=0.0, route_scale=1.0,
                             wg_shared_bits=_np(lay.shared_gate.view(torch.int16)).view(np.uint16).reshape(-1))
    ex = _mx_oracle(lay.experts, M.GATE_UP, 0.0)
    ref = M.moe_forward(_f32(x), ri, rw, ex, shared_expert=E, shared_weight=rsh)
    assert M.max_rel_err(_f32(out), ref) < TOL


def test_tiny_affine4_config_vs_oracle(dev):
    lay = S.make_layer("tiny", dev, seed=0)
    cfg = lay.cfg
    x = S.make_tokens(cfg["tokens"], cfg["H"], 0, dev)
    out = lay.layer(x)
    xb = F.f32_to_bf16_bits(_f32(x))
    _, ri, rw, _ = R.route(xb, _np(lay.gate_weight.view(torch.int16)).view(np.uint16), cfg["k"], R.SCORE_SOFTMAX_BF16,
                           norm_eps=0.0)
    a = lay.experts
    bits = lambda t: _np(t.view(torch.int16)).view(np.uint16)
    ex = M.Affine4Experts(_np(a.w13).view(np.uint32), bits(a.w13_scales), bits(a.w13_biases), _np(a.w2).view(np.uint32),
                          bits(a.w2_scales), bits(a.w2_biases), M.GATE_UP, 0.0, 64)
    ref = M.moe_forward(_f32(x), ri, rw, ex)
    assert M.max_rel_err(_f32(out), ref) < TOL


def test_batch_equals_tokens_one_at_a_time(dev, monkeypatch):
    # within one expert path: single tokens would otherwise take the CUDA-core weight
    # stream (its own two-token check is in test_gpu_stream.py)
    monkeypatch.setenv("WM_EXPERT_PATH", "mma")
    lay, x = _ds_case(dev, 12, 16, 1024, 256, seed=9)
    wts, idx = lay.layer.gate(x)
    full = W.experts_forward(x, idx, lay.experts, weights=wts, shared_expert=16, swiglu_limit=10.0)
    rows = [W.experts_forward(x[i:i + 1], idx[i:i + 1], lay.experts, weights=wts[i:i + 1], shared_expert=16,
                              swiglu_limit=10.0) for i in range(12)]
    assert torch.equal(full, torch.cat(rows, 0))
    un = W.experts_forward(x, idx, lay.experts, swiglu_limit=10.0)
    un1 = torch.cat([W.experts_forward(x[i:i + 1], idx[i:i + 1], lay.experts, swiglu_limit=10.0) for i in range(12)])
    assert torch.equal(un, un1)
    # route_reduce of the un-reduced output agrees with the fused combine
    routed_only = W.experts_forward(x, idx, lay.experts, weights=wts, swiglu_limit=10.0)
    assert M.max_rel_err(_f32(W.route_reduce(un, wts)), _f32(routed_only)) < TOL


def _affine_oracle(a):
    bits = lambda t: _np(t.view(torch.int16)).view(np.uint16)
    return M.Affine4Experts(_np(a.w13).view(np.uint32), bits(a.w13_scales), bits(a.w13_biases),
                            _np(a.w2).view(np.uint32), bits(a.w2_scales), bits(a.w2_biases), M.GATE_UP, 0.0, a.group)


@pytest.mark.parametrize("I", [320, 288, 352])
def test_cuda_core_rows_of_9_to_11_groups(dev, I):
    # down rows of I values are 9-11 scale groups of 32: the CUDA-core kernel splits each group over
    # 2 lanes there; every value of every group must be summed (I is not a multiple of 256, so both
    # formats take the CUDA-core path)
    T, E, k, H = 7, 6, 3, 512
    rng = np.random.default_rng(I)
    idx = torch.from_numpy(rng.integers(0, E, (T, k)).astype(np.int32)).to(dev)
    w = torch.from_numpy(rng.uniform(0.1, 1.0, (T, k)).astype(np.float32)).to(dev)
    x = S.make_tokens(T, H, I, dev)
    if I % 64 == 0:
        ex = S.make_affine4_experts(E, H, I, seed=I, device=dev)
        oracle = _affine_oracle(ex)
        out = W.experts_forward(x, idx, ex, weights=w)
    else:
        ex = S.make_mxfp4_experts(E, H, I, seed=I, device=dev)
        oracle = _mx_oracle(ex, M.UP_GATE, 10.0)
        out = W.experts_forward(x, idx, ex, weights=w, swiglu_limit=10.0)
    ref = M.moe_forward(_f32(x), _np(idx), _np(w), oracle)
    assert M.max_rel_err(_f32(out), ref) < TOL


@pytest.mark.parametrize("T", [1, 64, 300])
def test_affine4_tensor_core_path_vs_cuda_core_and_oracle(dev, T):
    # the tiny configuration's affine-4 experts (group 64) on the f16 tensor-core kernel (the default for
    # H, I multiples of 256) against the CUDA-core kernel (WM_EXPERT_PATH=simt) and the oracle; T = 300 takes
    # the prefill tile shape
    import os
    lay = S.make_layer("tiny", dev, seed=T + 1)
    x = S.make_tokens(T, 1024, T, dev)
    w, idx, _ = W.qwen_route(x, lay.gate_weight, 4, True)
    out_tc = W.experts_forward(x, idx, lay.experts, weights=w)
    old = os.environ.get("WM_EXPERT_PATH")
    os.environ["WM_EXPERT_PATH"] = "simt"
    try:
        out_cc = W.experts_forward(x, idx, lay.experts, weights=w)
    finally:
        if old is None:
            os.environ.pop("WM_EXPERT_PATH", None)
        else:
            os.environ["WM_EXPERT_PATH"] = old
    ref = M.moe_forward(_f32(x), _np(idx), _np(w), _affine_oracle(lay.experts))
    assert M.max_rel_err(_f32(out_tc), ref) < TOL
    assert M.max_rel_err(_f32(out_tc), _f32(out_cc)) < TOL
    un = W.experts_forward(x, idx, lay.experts)                       # un-reduced switch_mlp rows
    assert M.max_rel_err(_f32(un), M.switch_mlp(_f32(x), _np(idx), _affine_oracle(lay.experts))) < TOL


def test_route_reduce_and_rows_reduce_vs_float64(dev):
    # _route_reduce (model.py:502-504) on the device, and the slot-indexed form the expert-parallel
    # all-to-all layer uses: skipped slots, a float32 addend, float32 accumulation in j order
    rng = np.random.default_rng(31)
    T, k, H = 37, 9, 1024
    routed = torch.from_numpy(rng.normal(0, 1, (T, k, H)).astype(np.float32)).to(dev).to(torch.bfloat16)
    scores = torch.from_numpy(rng.uniform(0, 1, (T, k)).astype(np.float32)).to(dev)
    got = W.route_reduce(routed, scores)
    ref = (routed.double() * scores.double()[..., None]).sum(1)
    assert M.max_rel_err(_f32(got), ref.cpu().numpy()) < 1e-2
    R = 500
    y = torch.from_numpy(rng.normal(0, 1, (R, H)).astype(np.float32)).to(dev).to(torch.bfloat16)
    slots = torch.from_numpy(rng.integers(-2, R, (T, k)).astype(np.int32)).to(dev)
    add = torch.from_numpy(rng.normal(0, 1, (T, H)).astype(np.float32)).to(dev)
    from whallm_b200.moe import rows_reduce
    out = rows_reduce(y, slots, scores, add)
    s = slots.long().cpu()
    rows = torch.where((s >= 0)[..., None], y.double().cpu()[s.clamp(min=0)], torch.zeros((), dtype=torch.float64))
    ref2 = (rows * scores.double().cpu()[..., None]).sum(1) + add.double().cpu()
    assert M.max_rel_err(_f32(out), ref2.numpy()) < 1e-2


def _ws_layout(T, k, E, has_shared):
    """Offsets (bytes) of the grouping regions in the expert workspace (csrc/wm_moe.cuh carve_workspace)."""
    S = T * (k + has_shared)
    off, regions = 0, {}
    for name, nbytes in (("offsets", (E + 1) * 4), ("perm", S * 4), ("inv", S * 4), ("active", E * 4),
                         ("counters", 32), ("tiles", (E + S // 16 + 2) * 16)):
        regions[name] = (off, nbytes)
        off = (off + nbytes + 255) // 256 * 256
    return regions


@pytest.mark.parametrize("T,E,path", [(1, 16, "mma"), (3, 16, "mma"), (7, 257, "mma"), (2, 33, "stream"),
                                      (1, 513, "stream"), (7, 40, "stream")])
def test_in_kernel_grouping_equals_permute(dev, monkeypatch, T, E, path):
    # calls of at most 64 slots group their assignments inside the first expert kernel; the grouping it
    # writes to the workspace must be the permute kernel's (offsets, perm, inv, active list, counters and,
    # on the tensor path, the work list with the shared expert's tiles first)
    monkeypatch.setenv("WM_EXPERT_PATH", path)
    k, H, I = 8, 1024, 512
    ex = S.make_mxfp4_experts(E + 1, H, I, seed=T + E, device=dev)
    x = S.make_tokens(T, H, T, dev)
    rng = np.random.default_rng(T * E)
    ri = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    ri[0, 0] = ri[0, 1] if T > 1 else ri[0, 0]
    idx = torch.from_numpy(ri).to(dev)
    w = torch.full((T, k), 1.0 / k, device=dev)
    nbytes = W.experts.workspace_size(T, k, H, I, E + 1, True)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    W.experts_forward(x, idx, ex, weights=w, shared_expert=E, swiglu_limit=10.0, workspace=ws)
    torch.cuda.synchronize()
    lay = _ws_layout(T, k, E + 1, 1)
    get = lambda name, n: ws[lay[name][0]:lay[name][0] + 4 * n].view(torch.int32).cpu().numpy()
    ext = np.concatenate([ri, np.full((T, 1), E, np.int32)], axis=1)        # the shared slot is expert E
    r_off, r_perm, r_inv = M.permute(ext, E + 1)
    np.testing.assert_array_equal(get("offsets", E + 2), r_off)
    np.testing.assert_array_equal(get("perm", ext.size), r_perm)
    np.testing.assert_array_equal(get("inv", ext.size), r_inv)
    act = np.flatnonzero(np.diff(r_off) > 0).astype(np.int32)
    cnt = get("counters", 4)
    assert cnt[0] == act.size and cnt[1] == 0 and cnt[3] == 0
    np.testing.assert_array_equal(get("active", act.size), act)
    if path == "mma":
        tn = 32
        want = [(E, r_off[E] + q, min(tn, r_off[E + 1] - r_off[E] - q)) for q in range(0, r_off[E + 1] - r_off[E], tn)]
        for e in act:
            if e != E:
                n = r_off[e + 1] - r_off[e]
                want += [(e, r_off[e] + q, min(tn, n - q)) for q in range(0, n, tn)]
        assert cnt[2] == len(want)
        tiles = get("tiles", 4 * len(want)).reshape(-1, 4)[:, :3]
        np.testing.assert_array_equal(tiles, np.array(want, np.int32))


@pytest.mark.parametrize("path", ["mma", "stream"])
def test_small_call_invalid_id_gives_zeros(dev, monkeypatch, path):
    # a two-token call groups its slots in-kernel and combines in the down projection's last CTA:
    # an out-of-range id must still give zeros (and nothing outside the layer is read)
    monkeypatch.setenv("WM_EXPERT_PATH", path)
    E, H, I = 4, 256, 256
    ex = S.make_mxfp4_experts(E + 1, H, I, seed=3, device=dev)
    x = S.make_tokens(2, H, 3, dev)
    idx = torch.tensor([[0, 1, 2], [3, 0, 99]], dtype=torch.int32, device=dev)
    w = torch.full((2, 3), 0.25, device=dev)
    out = W.experts_forward(x, idx, ex, weights=w, shared_expert=E, swiglu_limit=10.0)
    assert torch.count_nonzero(out) == 0
    # and the next call on the same workspace is whole again (the grouping and the ticket are rewritten)
    idx_ok = torch.tensor([[0, 1, 2], [3, 0, 1]], dtype=torch.int32, device=dev)
    out2 = W.experts_forward(x, idx_ok, ex, weights=w, shared_expert=E, swiglu_limit=10.0)
    ref = M.moe_forward(_f32(x), _np(idx_ok), _np(w), _mx_oracle(ex, M.UP_GATE, 10.0), shared_expert=E)
    assert M.max_rel_err(_f32(out2), ref) < TOL


@pytest.mark.parametrize("path", ["mma", "stream"])
@pytest.mark.parametrize("T", [1, 2])
def test_small_call_repeats_bit_for_bit(dev, monkeypatch, path, T):
    # the fused combine's ticket is re-armed by every call: back-to-back calls give identical bits
    monkeypatch.setenv("WM_EXPERT_PATH", path)
    E, H, I, k = 12, 1024, 512, 6
    ex = S.make_mxfp4_experts(E + 1, H, I, seed=T, device=dev)
    x = S.make_tokens(T, H, T, dev)
    rng = np.random.default_rng(T)
    idx = torch.from_numpy(np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)).to(dev)
    w = torch.from_numpy(rng.uniform(0.1, 1.0, (T, k)).astype(np.float32)).to(dev)
    outs = [W.experts_forward(x, idx, ex, weights=w, shared_expert=E, swiglu_limit=10.0) for _ in range(4)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    ref = M.moe_forward(_f32(x), _np(idx), _np(w), _mx_oracle(ex, M.UP_GATE, 10.0), shared_expert=E)
    assert M.max_rel_err(_f32(outs[0]), ref) < TOL


def test_in_kernel_grouping_affine_tensor_path(dev):
    # 16 tokens of the tiny configuration (x top-4 = 64 slots) group their slots in the f16 gather kernel;
    # the grouping and the work list (64-token tiles, no shared expert) equal the permute kernel's
    lay = S.make_layer("tiny", dev, seed=2)
    cfg = lay.cfg
    T, k, E, H, I = 16, cfg["k"], cfg["E"], cfg["H"], cfg["I"]
    x = S.make_tokens(T, H, 2, dev)
    w, idx, _ = W.qwen_route(x, lay.gate_weight, k, True)
    nbytes = W.experts.workspace_size(T, k, H, I, E, False)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    out = W.experts_forward(x, idx, lay.experts, weights=w, workspace=ws)
    torch.cuda.synchronize()
    lay_ws = _ws_layout(T, k, E, 0)
    get = lambda name, n: ws[lay_ws[name][0]:lay_ws[name][0] + 4 * n].view(torch.int32).cpu().numpy()
    ri = _np(idx)
    r_off, r_perm, r_inv = M.permute(ri, E)
    np.testing.assert_array_equal(get("offsets", E + 1), r_off)
    np.testing.assert_array_equal(get("perm", ri.size), r_perm)
    np.testing.assert_array_equal(get("inv", ri.size), r_inv)
    want = []
    for e in range(E):
        n = r_off[e + 1] - r_off[e]
        want += [(e, r_off[e] + q, min(64, n - q)) for q in range(0, n, 64)]
    cnt = get("counters", 4)
    assert cnt[2] == len(want)
    np.testing.assert_array_equal(get("tiles", 4 * len(want)).reshape(-1, 4)[:, :3], np.array(want, np.int32))
    ref = M.moe_forward(_f32(x), ri, _np(w), _affine_oracle(lay.experts))
    assert M.max_rel_err(_f32(out), ref) < TOL
