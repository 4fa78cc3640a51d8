"""Pin the CPU oracle before trusting it (no GPU needed).

* MXFP4 quantizer == the reference's Swift known-answer tests, including the
  SHA-256 digests (DeepSeekRepackTests.swift:336-411, via mxfp4_kats.json).
* e2m1 rounding: vectorised form == literal restatement of fp4Code
  (MXFP4.swift:115-131) == fakequant._e2m1_round (fakequant.py:65-73).
* e4m3 encode/decode == ml_dtypes' float8_e4m3fn (the RNE conversion
  mx.to_fp8 performs after clipping).
* PackedRows write+read == fake_quant for all three formats (value-equal, as
  mx.array_equal checks) and uses less memory than bf16 (test_v41_packed_cache.py:12-26).
* FP8 row dequant == dequant_fp8-style reference (test_deepseek_v41.py:129-155).
* Router oracle: exp/log accuracy, top-k == fp64 top-k, positional ties
  (test_runtime.py:2530-2533), permutation == stable argsort.
* Golden fixtures regenerate identically from the oracle.
"""
import hashlib
import json
import os

import ml_dtypes
import numpy as np
import pytest

from oracle import formats as F
from oracle import moe as M
from oracle import router as R

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _kats():
    with open(os.path.join(GOLD, "mxfp4_kats.json")) as f:
        return json.load(f)


def test_mxfp4_fixed_vector_kat():
    k = _kats()["fixed_vector"]
    vals = np.array(k["values"], np.float32)
    bits = (vals.view(np.uint32) >> 16).astype(np.uint16).reshape(1, 32)
    w, s = F.mxfp4_quantize_bf16(bits)
    assert list(w.reshape(-1)) == k["weights"]
    assert list(s.reshape(-1)) == k["scales"]


def test_mxfp4_bf16_rows_kat():
    k = _kats()["bf16_rows"]
    w, s = F.mxfp4_quantize_bf16(np.array(k["bits"], np.uint16).reshape(2, 32))
    assert list(w.reshape(-1)) == k["weights"]
    assert list(s.reshape(-1)) == k["scales"]


def test_mxfp4_fp8_blocks_kat():
    k = _kats()["fp8_blocks"]
    src = np.array(k["first_row"] + [0] * (127 * 128), np.uint8)
    inv = np.frombuffer(bytes(k["inverse_scale_bytes"]), np.uint16)
    w, s = F.mxfp4_quantize_fp8(src, inv, 128, 128)
    assert list(w.reshape(-1)[:16]) == k["weights_prefix"]
    assert list(s.reshape(-1)[:4]) == k["scales_prefix"]


def test_mxfp4_fp8_sha256_kat():
    k = _kats()["fp8_sha256"]
    i = np.arange(k["rows"] * k["cols"])
    v = ((i * k["mul"] + k["add"]) & 0xFF).astype(np.uint8)
    v = np.where((v & 0x7F) == 0x7F, v ^ 1, v).astype(np.uint8)
    w, s = F.mxfp4_quantize_fp8(v, np.frombuffer(bytes(k["inverse_scale_bytes"]), np.uint16), 128, 128)
    assert hashlib.sha256(w.tobytes()).hexdigest() == k["weights_sha256"]
    assert hashlib.sha256(s.tobytes()).hexdigest() == k["scales_sha256"]


def test_e2m1_code_matches_literal_loop_and_fakequant():
    rng = np.random.default_rng(3)
    mids = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 7.0]
    v = np.concatenate([rng.normal(0, 3, 3000), mids, [-m for m in mids], [0.0, -0.0]]).astype(np.float32)
    codes = F.e2m1_code(v)
    assert all(codes[i] == F.e2m1_code_loop(v[i]) for i in range(len(v)))
    mag = F.E2M1[codes & 7]
    assert np.array_equal(mag, np.abs(F.e2m1_round(np.clip(v, -6, 6))))


def test_e4m3_matches_ml_dtypes():
    rng = np.random.default_rng(4)
    x = np.concatenate([rng.normal(0, 100, 50000), rng.normal(0, 1e-2, 50000), rng.uniform(-448, 448, 20000),
                        [0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -11, 2.0 ** -6]]).astype(np.float32)
    x = np.clip(x, -448, 448)
    assert np.array_equal(F.f32_to_e4m3(x), x.astype(ml_dtypes.float8_e4m3fn).view(np.uint8))
    codes = np.arange(256, dtype=np.uint8)
    assert np.array_equal(F.e4m3_to_f32(codes), codes.view(ml_dtypes.float8_e4m3fn).astype(np.float32),
                          equal_nan=True)


@pytest.mark.parametrize("kind", ["fp4_e4m3", "fp4_ue8m0", "fp8_ue8m0"])
def test_packed_rows_round_trip_equals_fake_quant(kind):
    rng = np.random.default_rng(941)
    value = F.round_bf16((rng.normal(0, 1, (1, 23, 64)) * 2.3).astype(np.float32))
    fmt = F.PACKED_KIND_TO_FMT[kind]
    payload, scales = F.kv_quantize(value, fmt)
    got = F.round_bf16(F.kv_dequantize(payload, scales, fmt, 64))
    expected = F.round_bf16(F.fake_quant(value, kind))
    # value equality as mx.array_equal checks it (-0.0 == +0.0): the packed form
    # stores +0 where the fake-quant keeps the sign of a value rounded to zero
    assert np.array_equal(got, expected)
    assert payload.nbytes + scales.nbytes < value.size * 2


def test_fp8_rows_dequant_matches_blockwise_reference():
    rng = np.random.default_rng(7)
    raw = rng.integers(0, 256, size=(64, 64), dtype=np.uint8)
    raw[raw % 128 == 127] = 0
    scale = rng.integers(122, 133, size=(64, 2), dtype=np.uint8)
    got = F.kv_dequantize(raw, scale, F.KV_MXFP8_B32, 64)
    ref = F.e4m3_to_f32(raw).reshape(64, 2, 32) * F.e8m0_to_f32(scale)[..., None]
    np.testing.assert_array_equal(got, ref.reshape(64, 64))


def test_fp32_block64_format_and_zero_block():
    x = np.zeros((2, 128), np.float32)
    x[0, :64] = F.round_bf16(np.linspace(-3, 3, 64).astype(np.float32))
    p, s = F.kv_quantize(x, F.KV_FP8_F32_B64)
    assert s.dtype == np.float32 and s.shape == (2, 2)
    assert s[0, 0] == np.float32(3.0) / np.float32(448.0) and s[0, 1] == 0 and s[1, 0] == 0
    assert not p[0, 64:].any() and not p[1].any()
    d = F.kv_dequantize(p, s, F.KV_FP8_F32_B64, 128)
    assert np.max(np.abs(d[0, :64] - x[0, :64])) <= 3.0 / 16


def test_mxfp4_dequant_exact_and_code8_positive_zero():
    packed = np.array([[0x98] + [0] * 15], np.uint8)
    scales = np.array([[127]], np.uint8)
    d = F.mxfp4_dequantize(packed, scales)
    assert d[0, 0] == 0.0 and not np.signbit(d[0, 0]) and d[0, 1] == -0.5
    s0 = F.mxfp4_dequantize(np.array([[0x77] * 16], np.uint8), np.array([[0]], np.uint8))
    assert s0[0, 0] == np.float32(6.0 * 2.0 ** -127)


def test_exp_and_softplus_accuracy():
    x = np.random.default_rng(1).uniform(-87, 88.7, 200000).astype(np.float32)
    y = R.exp_f32(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    assert np.max(np.abs(y - ref) / ref) < 2.0 ** -22
    v = np.random.default_rng(2).normal(0, 5, 100000).astype(np.float32)
    sp = R.softplus_f32(v).astype(np.float64)
    assert np.max(np.abs(sp - np.logaddexp(v.astype(np.float64), 0)) / np.logaddexp(v.astype(np.float64), 0)) < 1e-6


def test_router_topk_matches_fp64_and_renormalises():
    rng = np.random.default_rng(5)
    T, H, E, k = 32, 1024, 128, 8
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    logits, idx, w, _ = R.route(xb, wb, k, R.SCORE_SOFTMAX, norm_eps=0.0)
    ref = F.bf16_bits_to_f32(xb).astype(np.float64) @ F.bf16_bits_to_f32(wb).astype(np.float64).T
    assert np.max(np.abs(logits - ref)) < 1e-5
    assert np.array_equal(idx, np.argsort(-ref, axis=1, kind="stable")[:, :k])
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)
    p = np.exp(ref - ref.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    sel = np.take_along_axis(p, idx, 1)
    np.testing.assert_allclose(w, sel / sel.sum(1, keepdims=True), rtol=1e-5)


def test_router_v41_semantics_bias_selects_but_does_not_scale():
    rng = np.random.default_rng(6)
    T, H, E, k = 8, 256, 32, 4
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    bias = np.zeros(E, np.float32)
    bias[7] = 100.0
    logits, idx, w, _ = R.route(xb, wb, k, R.SCORE_SQRTSOFTPLUS, select_bias=bias, norm_eps=1e-20, route_scale=1.5)
    assert (idx[:, 0] == 7).all()
    score = np.sqrt(np.logaddexp(logits.astype(np.float64), 0))
    sel = np.take_along_axis(score, idx, 1)
    np.testing.assert_allclose(w, 1.5 * sel / (sel.sum(1, keepdims=True) + 1e-20), rtol=1e-5)


def test_stable_topk_ties_by_position():
    assert R.stable_topk_indices(np.array([[1.0, 1.0, 1.0, 0.5]]), 2).tolist() == [[0, 1]]
    xb = np.zeros((1, 256), np.uint16)
    wb = np.zeros((8, 256), np.uint16)
    _, idx, _, _ = R.route(xb, wb, 3, R.SCORE_NONE)
    assert idx.tolist() == [[0, 1, 2]]


def test_permute_is_stable_argsort():
    rng = np.random.default_rng(8)
    idx = rng.integers(0, 16, (50, 4)).astype(np.int32)
    off, perm, inv = M.permute(idx, 16)
    flat = idx.reshape(-1)
    assert np.array_equal(perm, np.argsort(flat, kind="stable"))
    assert np.array_equal(inv[perm], np.arange(flat.size))
    assert np.array_equal(np.diff(off), np.bincount(flat, minlength=16))


def test_golden_fixtures_regenerate(tmp_path):
    from tests.golden import make_golden as G
    out = tmp_path / "g.npz"
    G.make_golden(str(out))
    a = np.load(os.path.join(GOLD, "golden.npz"))
    b = np.load(out)
    assert set(a.files) == set(b.files)
    for n in a.files:
        assert np.array_equal(a[n], b[n], equal_nan=True), n


def _bf16_round(a):
    import ml_dtypes
    return np.asarray(a, np.float32).astype(ml_dtypes.bfloat16).astype(np.float32)


def _butterfly32(part):
    a = part.astype(np.float32)
    lanes = np.arange(32)
    for m in (16, 8, 4, 2, 1):
        a = (a + a[:, lanes ^ m]).astype(np.float32)
    return a[:, 0]


@pytest.mark.parametrize("T,H,E,k", [(64, 2048, 512, 10), (33, 1024, 16, 4), (7, 512, 100, 3)])
def test_router_bf16_gate_follows_the_reference_dtypes(T, H, E, k):
    """SCORE_SOFTMAX_BF16 against a numpy restatement of the Qwen gate's dtypes
    (qwen4_exp.py:683, 693-699): bf16 logits, float32 softmax rounded to bf16
    (ml_dtypes, round-to-nearest-even), top-k of the bf16 probabilities with
    ties to the lower id, weights bf16(p / bf16(sum)), shared gate
    bf16(sigmoid(bf16 logit)).  The float32 steps use the oracle's own exp and
    summation order, so the comparison is exact."""
    rng = np.random.default_rng(T + E)
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    sg = F.f32_to_bf16_bits((rng.normal(0, 1, (H,)) / np.sqrt(H)).astype(np.float32))
    lb = rng.normal(0, 1, E).astype(np.float32)
    logits, idx, w, sh = R.route(xb, wb, k, R.SCORE_SOFTMAX_BF16, logit_bias=lb, norm_eps=0.0, wg_shared_bits=sg)
    l32, _, _, sh32 = R.route(xb, wb, k, R.SCORE_SOFTMAX, logit_bias=lb, norm_eps=0.0, wg_shared_bits=sg)
    assert np.array_equal(logits.view(np.uint32), l32.view(np.uint32))     # the float32 gate output, biased
    z = _bf16_round(logits)
    e = R.exp_f32(z - z.max(1, keepdims=True)).reshape(T, E)
    part = np.zeros((T, 32), np.float32)
    for j in range(0, E, 32):
        blk = np.zeros((T, 32), np.float32)
        blk[:, :min(32, E - j)] = e[:, j:j + 32]
        part = (part + blk).astype(np.float32)
    p = _bf16_round(e / _butterfly32(part)[:, None])
    order = np.lexsort((np.broadcast_to(np.arange(E), p.shape), -p), axis=-1)[:, :k]
    np.testing.assert_array_equal(idx, order)
    sel = np.take_along_axis(p, idx, 1)
    s = np.zeros(T, np.float32)
    for j in range(k):
        s = (s + sel[:, j]).astype(np.float32)
    np.testing.assert_array_equal(w.view(np.uint32), _bf16_round(sel / _bf16_round(s)[:, None]).view(np.uint32))
    assert not np.any(w.view(np.uint32) & 0xffff)                          # bf16 values
    g = _bf16_round(np.log(sh32 / (1 - sh32)))                               # the float32 shared logit, rounded
    assert np.max(np.abs(sh - _bf16_round(1 / (1 + np.exp(-g.astype(np.float64)))))) <= 2.0 ** -8


def test_router_bf16_gate_ties_go_to_the_lower_id():
    # 40 equal logits: equal bf16 probabilities, the first k ids win; weights 1/k in bf16
    xb = np.zeros((2, 256), np.uint16)
    wb = np.zeros((40, 256), np.uint16)
    _, idx, w, _ = R.route(xb, wb, 5, R.SCORE_SOFTMAX_BF16, norm_eps=0.0)
    assert idx.tolist() == [[0, 1, 2, 3, 4]] * 2
    assert np.all(w == _bf16_round(np.float32(0.2)))


def test_host_mxfp4_quantizer_equals_the_numpy_restatement():
    # the C quantizer the CPU baseline builds its layers with gives the bytes of formats.mxfp4_quantize_values
    from oracle import synthetic as SY
    rng = np.random.default_rng(12)
    v = F.round_bf16(rng.normal(0, 0.02, (64, 512)).astype(np.float32))
    v[0, :32] = 0.0                                                  # all-zero group
    v[1, :32] *= np.float32(1e-30)                                   # tiny scales (clamped exponent)
    v[2, :32] = np.float32(6.0) * np.float32(2.0 ** 100)             # huge values
    v[3, 32:64] = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, -0.25] * 4, np.float32)   # e2m1 ties
    v[4, :32] = -0.0
    p, s = SY.mxfp4_quantize(v)
    rp, rs = F.mxfp4_quantize_values(v)
    np.testing.assert_array_equal(p, rp)
    np.testing.assert_array_equal(s, rs)


def test_host_normal_generator_is_seeded_bf16_normal():
    from oracle import synthetic as SY
    a = SY.normal_bf16(3, 5, (1000, 1001), 0.02)
    b = SY.normal_bf16(3, 5, (1000, 1001), 0.02)
    c = SY.normal_bf16(3, 6, (1000, 1001), 0.02)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert np.array_equal(a, F.round_bf16(a))
    assert abs(float(a.mean())) < 1e-4 and abs(float(a.std()) - 0.02) < 1e-4


# Blocks for the OCP Microscaling Formats (MX) Specification v1.0 conversion to MXFP8 E4M3: shared
# exponent X = floor(log2 max|V|) - 8, E8M0 byte X + 127, elements V / 2^X rounded to nearest even in
# E4M3 and saturated at +-448.
_MX8 = [[448.0], [1.0], [500.0, 1.0], [512.0, -3.0], [0.75, 0.0078125], [6.0, 1.0625], [3.0e-5, -1.0e-6]]


def _e4m3(v):
    return int(F.f32_to_e4m3(np.array([v], np.float32))[0])


def test_mxfp8_rule_follows_the_ocp_mx_conversion():
    from oracle.formats import kv_quantize, KV_MXFP8_B32
    for vals in _MX8:
        block = np.zeros(32, np.float32)
        block[:len(vals)] = vals
        p, s = kv_quantize(block[None], KV_MXFP8_B32)
        amax = float(np.max(np.abs(block)))
        X = int(np.floor(np.log2(amax))) - 8
        assert int(s[0, 0]) == X + 127
        for i, v in enumerate(vals):
            assert int(p[0, i]) == _e4m3(np.clip(v / 2.0 ** X, -448, 448)), (vals, i)


def test_mxfp8_rule_hand_checked_codes():
    # codes written out from the E4M3 layout (sign, 4 exponent bits with bias 7, 3 mantissa bits)
    cases = [([448.0], 127, {0: 0x7E}), ([1.0], 119, {0: 0x78}), ([500.0, 1.0], 127, {0: 0x7E, 1: 0x38}),
             ([512.0, -3.0], 128, {0: 0x78, 1: 0xBC}),
             ([6.0, 1.0625], 121, {0: 0x7C, 1: 0x68}),     # 1.0625 * 2^6: a tie between 1.0 and 1.125 -> 1.0
             ([0.0] * 32, 0, {0: 0x00, 31: 0x00})]
    from oracle.formats import kv_quantize, KV_MXFP8_B32
    for vals, byte, codes in cases:
        block = np.zeros(32, np.float32)
        block[:len(vals)] = vals
        p, s = kv_quantize(block[None], KV_MXFP8_B32)
        assert int(s[0, 0]) == byte, vals
        for i, c in codes.items():
            assert int(p[0, i]) == c, (vals, i, hex(int(p[0, i])))


def test_mxfp8_scale_byte_clamps_and_ties_round_to_even():
    from oracle.formats import kv_quantize, KV_MXFP8_B32
    # max 2^-130 (a float32 subnormal): floor(log2) - 8 = -138 clamps to the smallest E8M0 exponent -127
    block = np.zeros(32, np.float32)
    block[0] = np.float32(2.0 ** -130)
    _, s = kv_quantize(block[None], KV_MXFP8_B32)
    assert int(s[0, 0]) == 0
    # max 256 (X = 0): 1.0625 lies halfway between the E4M3 values 1.0 and 1.125 -> the even code (1.0)
    block = np.zeros(32, np.float32)
    block[:3] = [256.0, 1.0625, 1.1875]
    p, s = kv_quantize(block[None], KV_MXFP8_B32)
    assert int(s[0, 0]) == 127
    assert int(p[0, 1]) == 0x38 and int(p[0, 2]) == 0x3A   # 1.1875 halfway between 1.125 and 1.25 -> 1.25
