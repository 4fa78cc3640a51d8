"""Device router vs the CPU oracle: indices and weights bit-exact.

Covers every score function, logit and selection biases, the renormalisation
variants (V4.1 eps 1e-20 x 1.5, Qwen plain sum, none), the Qwen shared-expert
gate, exact ties (positional rule, test_runtime.py:2530-2533), E not a
multiple of 32, T = 0 and k = 1, and the DeepSeek-class shapes.
"""
import os

import numpy as np
import pytest
import torch

import whallm_b200 as W
from oracle import formats as F
from oracle import router as R

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
FN = {R.SCORE_SOFTMAX: "softmax", R.SCORE_SIGMOID: "sigmoid", R.SCORE_SQRTSOFTPLUS: "sqrtsoftplus", R.SCORE_NONE: "none",
      R.SCORE_SOFTMAX_BF16: "softmax_bf16"}


def _bf16(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(torch.bfloat16).to(dev)


def _run(dev, xb, wb, k, fn, lb=None, sb=None, eps=-1.0, scale=1.0, sg=None):
    x = _bf16(xb, dev)
    w = _bf16(wb, dev)
    t = lambda a: None if a is None else torch.from_numpy(a).to(dev)
    logits = torch.empty(xb.shape[0], wb.shape[0], dtype=torch.float32, device=dev)
    wts, idx, sh = W.route(x, w, k, FN[fn], logit_bias=t(lb), select_bias=t(sb), norm_eps=None if eps < 0 else eps,
                           route_scale=scale, shared_gate=None if sg is None else _bf16(sg, dev), logits_out=logits)
    return (logits.cpu().numpy(), idx.cpu().numpy(), wts.cpu().numpy(),
            None if sh is None else sh.reshape(-1).cpu().numpy())


def _check(got, ref):
    lg, idx, w, sh = got
    rl, ri, rw, rs = ref
    np.testing.assert_array_equal(lg.view(np.uint32), rl.view(np.uint32))
    np.testing.assert_array_equal(idx, ri)
    np.testing.assert_array_equal(w.view(np.uint32), rw.view(np.uint32))
    if rs is not None:
        np.testing.assert_array_equal(sh.view(np.uint32), rs.view(np.uint32))


@pytest.mark.parametrize("case", range(4))
def test_router_golden(dev, case):
    g = np.load(os.path.join(GOLD, "golden.npz"))
    cases = [(R.SCORE_SOFTMAX, None, "rt_logit_bias", 0.0, 1.0, "rt_shared_gate"),
             (R.SCORE_SIGMOID, "rt_sel_bias", None, 1e-20, 2.5, None),
             (R.SCORE_SQRTSOFTPLUS, "rt_sel_bias", "rt_logit_bias", 1e-20, 1.5, None),
             (R.SCORE_NONE, None, None, -1.0, 1.0, None)]
    fn, sb, lb, eps, scale, sg = cases[case]
    got = _run(dev, g["rt_x"], g["rt_w"], 6, fn, None if lb is None else g[lb], None if sb is None else g[sb], eps,
               scale, None if sg is None else g[sg])
    ref = (g[f"rt{case}_logits"], g[f"rt{case}_idx"], g[f"rt{case}_w"],
           g[f"rt{case}_shared"] if f"rt{case}_shared" in g.files else None)
    _check(got, ref)


@pytest.mark.parametrize("fn", [R.SCORE_SOFTMAX, R.SCORE_SIGMOID, R.SCORE_SQRTSOFTPLUS, R.SCORE_SOFTMAX_BF16])
@pytest.mark.parametrize("shape", [(1, 7168, 256, 8), (37, 2048, 512, 10), (5, 1024, 16, 4), (9, 264, 100, 1),
                                   (300, 7168, 256, 8), (129, 2056, 33, 3)])
def test_router_random_vs_oracle(dev, fn, shape):
    T, H, E, k = shape
    rng = np.random.default_rng(T * 131 + E + fn)
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    lb = np.log(np.arange(1, E + 1, dtype=np.float64) ** -1.0 / np.sum(np.arange(1, E + 1) ** -1.0)).astype(np.float32)
    rng.shuffle(lb)
    sb = rng.normal(0, 0.1, E).astype(np.float32)
    ref = R.route(xb, wb, k, fn, logit_bias=lb, select_bias=sb, norm_eps=1e-20, route_scale=1.5)
    _check(_run(dev, xb, wb, k, fn, lb, sb, 1e-20, 1.5), ref)


def test_router_exact_ties_choose_lower_index(dev):
    xb = np.zeros((3, 256), np.uint16)
    wb = np.zeros((40, 256), np.uint16)
    ref = R.route(xb, wb, 5, R.SCORE_SOFTMAX, norm_eps=0.0)
    got = _run(dev, xb, wb, 5, R.SCORE_SOFTMAX, eps=0.0)
    _check(got, ref)
    assert got[1].tolist() == [[0, 1, 2, 3, 4]] * 3
    s = torch.tensor([[1.0, 1.0, 1.0, 0.5]], device=dev)
    assert W.stable_topk_indices(s, 2).cpu().tolist() == [[0, 1]]


def test_router_empty_batch(dev):
    x = torch.empty(0, 256, dtype=torch.bfloat16, device=dev)
    w = torch.zeros(16, 256, dtype=torch.bfloat16, device=dev)
    wts, idx, _ = W.route(x, w, 4)
    assert wts.shape == (0, 4) and idx.shape == (0, 4)


def test_gate_v41_semantics(dev):
    rng = np.random.default_rng(77)
    T, H, E, k = 16, 512, 64, 6
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    bias = rng.normal(0, 0.5, E).astype(np.float32)
    gate = W.Gate(_bf16(wb, dev), k, "sqrtsoftplus", bias=torch.from_numpy(bias).to(dev), route_scale=1.5)
    wts, idx = gate(_bf16(xb, dev))
    _, ri, rw, _ = R.route(xb, wb, k, R.SCORE_SQRTSOFTPLUS, select_bias=bias, norm_eps=1e-20, route_scale=1.5)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_array_equal(wts.cpu().numpy().view(np.uint32), rw.view(np.uint32))


@pytest.mark.parametrize("T", [1, 32, 300, 4096])
def test_qwen_bf16_gate_vs_oracle(dev, T):
    """The Qwen gate in the reference's dtypes (bf16 logits, bf16 probabilities,
    bf16 renormalisation, bf16 shared gate) at the Qwen-class shape, E = 512,
    top-10, Zipf 1.1 logit bias: indices, weights and shared weights bit-exact."""
    H, E, k = 2048, 512, 10
    rng = np.random.default_rng(T + 1)
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    sg = F.f32_to_bf16_bits((rng.normal(0, 1, (H,)) / np.sqrt(H)).astype(np.float32))
    lb = np.log(np.arange(1, E + 1, dtype=np.float64) ** -1.1 / np.sum(np.arange(1, E + 1) ** -1.1)).astype(np.float32)
    rng.shuffle(lb)
    ref = R.route(xb, wb, k, R.SCORE_SOFTMAX_BF16, logit_bias=lb, norm_eps=0.0, wg_shared_bits=sg)
    _check(_run(dev, xb, wb, k, R.SCORE_SOFTMAX_BF16, lb, None, 0.0, 1.0, sg), ref)


def test_qwen_route_uses_the_bf16_gate(dev):
    rng = np.random.default_rng(3)
    T, H, E, k = 16, 512, 64, 6
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    sg = F.f32_to_bf16_bits((rng.normal(0, 1, (H,)) / np.sqrt(H)).astype(np.float32))
    w, idx, sh = W.qwen_route(_bf16(xb, dev), _bf16(wb, dev), k, True, shared_gate=_bf16(sg, dev))
    _, ri, rw, rs = R.route(xb, wb, k, R.SCORE_SOFTMAX_BF16, norm_eps=0.0, wg_shared_bits=sg)
    np.testing.assert_array_equal(idx.cpu().numpy(), ri)
    np.testing.assert_array_equal(w.cpu().numpy().view(np.uint32), rw.view(np.uint32))
    np.testing.assert_array_equal(sh.reshape(-1).cpu().numpy().view(np.uint32), rs.view(np.uint32))


def test_bf16_gate_exact_ties_choose_lower_index(dev):
    xb = np.zeros((3, 256), np.uint16)
    wb = np.zeros((40, 256), np.uint16)
    ref = R.route(xb, wb, 5, R.SCORE_SOFTMAX_BF16, norm_eps=0.0)
    got = _run(dev, xb, wb, 5, R.SCORE_SOFTMAX_BF16, eps=0.0)
    _check(got, ref)
    assert got[1].tolist() == [[0, 1, 2, 3, 4]] * 3


@pytest.mark.parametrize("fn", [R.SCORE_SOFTMAX, R.SCORE_SOFTMAX_BF16, R.SCORE_SIGMOID, R.SCORE_SQRTSOFTPLUS, R.SCORE_NONE])
@pytest.mark.parametrize("shape", [(3, 1024, 200, 20), (5, 512, 1000, 32), (2, 256, 129, 1), (64, 2048, 513, 10)])
def test_wide_router_cta_kernel_vs_oracle(dev, fn, shape):
    # E > 128 runs one CTA per token: ragged E, k up to 32, every score function, bit-exact
    T, H, E, k = shape
    rng = np.random.default_rng(T * 7 + E + fn)
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    sb = rng.normal(0, 0.1, E).astype(np.float32)
    eps = -1.0 if fn == R.SCORE_NONE else 1e-20
    ref = R.route(xb, wb, k, fn, select_bias=sb, norm_eps=eps, route_scale=1.5)
    _check(_run(dev, xb, wb, k, fn, None, sb, eps, 1.5), ref)


def test_wide_router_exact_ties_choose_lower_index(dev):
    # 300 equal logits: every warp's list and the merge must take ids 0..k-1
    xb = np.zeros((2, 256), np.uint16)
    wb = np.zeros((300, 256), np.uint16)
    for fn in (R.SCORE_SOFTMAX, R.SCORE_SOFTMAX_BF16):
        ref = R.route(xb, wb, 12, fn, norm_eps=0.0)
        got = _run(dev, xb, wb, 12, fn, eps=0.0)
        _check(got, ref)
        assert got[1].tolist() == [list(range(12))] * 2


@pytest.mark.parametrize("fn", [R.SCORE_SOFTMAX, R.SCORE_SOFTMAX_BF16, R.SCORE_SIGMOID])
@pytest.mark.parametrize("E,k", [(700, 20), (513, 10), (1024, 32), (257, 8)])
def test_wide_router_cross_warp_ties(dev, fn, E, k):
    # gate rows drawn from 6 distinct rows: equal logits spread over every warp of the CTA, so the
    # per-warp winners tie with each other and the merge alone decides by expert id
    rng = np.random.default_rng(E + k + fn)
    base = (rng.normal(0, 1, (6, 512)) / np.sqrt(512)).astype(np.float32)
    wb = F.f32_to_bf16_bits(base[rng.integers(0, 6, E)])
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (3, 512)).astype(np.float32))
    ref = R.route(xb, wb, k, fn, norm_eps=1e-20)
    _check(_run(dev, xb, wb, k, fn, eps=1e-20), ref)


@pytest.mark.parametrize("fn", [R.SCORE_SIGMOID, R.SCORE_SQRTSOFTPLUS, R.SCORE_NONE])
@pytest.mark.parametrize("E", [100, 513])
def test_router_nan_and_inf_logits(dev, fn, E):
    # token 0 holds +inf: its logits are +-inf where the gate column is nonzero and NaN where it is zero;
    # NaN keys sort as -inf (lowest id first among them), on the warp and on the CTA kernel
    rng = np.random.default_rng(E + fn)
    x = rng.normal(0, 1, (2, 256)).astype(np.float32)
    x[0, 5] = np.inf
    w = (rng.normal(0, 1, (E, 256)) / 16).astype(np.float32)
    w[::3, 5] = 0.0
    xb, wb = F.f32_to_bf16_bits(x), F.f32_to_bf16_bits(w)
    eps = -1.0 if fn == R.SCORE_NONE else 1e-20
    lg, idx, wt, _ = _run(dev, xb, wb, 6, fn, eps=eps)
    rl, ri, rw, _ = R.route(xb, wb, 6, fn, norm_eps=eps)
    assert np.isnan(rl[0]).any() and np.isinf(rl[0]).any()
    np.testing.assert_array_equal(lg, rl)           # NaN-aware: NaN payloads may differ host to device
    np.testing.assert_array_equal(idx, ri)
    np.testing.assert_array_equal(wt, rw)


@pytest.mark.parametrize("fn", [R.SCORE_SOFTMAX, R.SCORE_SOFTMAX_BF16, R.SCORE_SQRTSOFTPLUS])
@pytest.mark.parametrize("shape", [(65, 2048, 513, 10), (200, 264, 40, 4), (1000, 4096, 256, 8), (77, 1032, 129, 6)])
def test_many_token_short_row_logits_vs_oracle(dev, fn, shape):
    # T > 64 with H <= 4096 takes the bit-reversed tree kernel: logits, routes and weights bit-exact,
    # including rows that end inside a 256-column block and tiles past E and T
    T, H, E, k = shape
    rng = np.random.default_rng(T + H + E)
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    sg = F.f32_to_bf16_bits((rng.normal(0, 1, (H,)) / np.sqrt(H)).astype(np.float32))
    lb = rng.normal(0, 1, E).astype(np.float32)
    ref = R.route(xb, wb, k, fn, logit_bias=lb, norm_eps=0.0, wg_shared_bits=sg)
    _check(_run(dev, xb, wb, k, fn, lb, None, 0.0, 1.0, sg), ref)


@pytest.mark.parametrize("fn", [R.SCORE_SOFTMAX, R.SCORE_SIGMOID, R.SCORE_SQRTSOFTPLUS, R.SCORE_NONE,
                                R.SCORE_SOFTMAX_BF16])
@pytest.mark.parametrize("shape", [(1, 1024, 8, 2), (3, 264, 32, 5), (70, 512, 31, 4), (64, 1024, 16, 4)])
def test_small_gates_vs_oracle(dev, fn, shape):
    # up to 32 gate rows (a shared gate on the 31-expert case fills the 32nd), every score function with
    # logit and selection biases, token counts not a multiple of the top-k kernel's 4 tokens per CTA
    T, H, E, k = shape
    rng = np.random.default_rng(T + E + fn)
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    lb = rng.normal(0, 0.5, E).astype(np.float32)
    sb = rng.normal(0, 0.1, E).astype(np.float32)
    sg = F.f32_to_bf16_bits((rng.normal(0, 1, (H,)) / np.sqrt(H)).astype(np.float32)) if E == 31 else None
    eps = -1.0 if fn == R.SCORE_NONE else 1e-20
    ref = R.route(xb, wb, k, fn, logit_bias=lb, select_bias=sb, norm_eps=eps, route_scale=1.5, wg_shared_bits=sg)
    _check(_run(dev, xb, wb, k, fn, lb, sb, eps, 1.5, sg), ref)


@pytest.mark.parametrize("fn", [R.SCORE_SOFTMAX_BF16, R.SCORE_SQRTSOFTPLUS])
def test_many_tokens_wide_tree_tiles_vs_oracle(dev, fn):
    # 5000 tokens x (512 experts + a shared gate) on short rows: two waves of 8 x 4 output tiles per thread;
    # ragged rows (513 of 128 per CTA), tokens (5000 of 64) and row length (1032 of 256)
    T, H, E, k = 5000, 1032, 512, 6
    rng = np.random.default_rng(fn + 5)
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    sg = F.f32_to_bf16_bits((rng.normal(0, 1, (H,)) / np.sqrt(H)).astype(np.float32))
    lb = rng.normal(0, 0.5, E).astype(np.float32)
    ref = R.route(xb, wb, k, fn, logit_bias=lb, norm_eps=1e-20, wg_shared_bits=sg)
    _check(_run(dev, xb, wb, k, fn, lb, None, 1e-20, 1.0, sg), ref)
