"""Device number formats vs the CPU oracle and the golden fixtures: bit-exact.

MXFP4 quantize (Swift KATs + random + edge groups), MXFP4 dequant, affine-4
quantize/dequant, every KV row format (payload, scales, dequant), gather.
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import whallm_b200 as W
from oracle import formats as F

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _bf16(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16).to(dev)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def test_mxfp4_quantize_kats(dev):
    k = json.load(open(os.path.join(GOLD, "mxfp4_kats.json")))
    fv = k["fixed_vector"]
    vals = np.array(fv["values"], np.float32)
    p, s = W.mxfp4_quantize(_bf16((vals.view(np.uint32) >> 16).astype(np.uint16).reshape(1, 32), dev))
    assert p.cpu().numpy().reshape(-1).tolist() == fv["weights"]
    assert s.cpu().numpy().reshape(-1).tolist() == fv["scales"]
    br = k["bf16_rows"]
    p, s = W.mxfp4_quantize(_bf16(np.array(br["bits"], np.uint16).reshape(2, 32), dev))
    assert p.cpu().numpy().reshape(-1).tolist() == br["weights"]
    assert s.cpu().numpy().reshape(-1).tolist() == br["scales"]
    # the SHA-256 KAT through the bf16 values the FP8 conversion produces
    kk = k["fp8_sha256"]
    i = np.arange(128 * 128)
    v = ((i * kk["mul"] + kk["add"]) & 0xFF).astype(np.uint8)
    v = np.where((v & 0x7F) == 0x7F, v ^ 1, v).astype(np.uint8)
    inv = F.bf16_bits_to_f32(np.frombuffer(bytes(kk["inverse_scale_bytes"]), np.uint16))[0]
    vals = F.round_bf16((F.e4m3_to_f32(v) * inv).astype(np.float32)).reshape(128, 128)
    p, s = W.mxfp4_quantize(_bf16(F.f32_to_bf16_bits(vals), dev))
    assert hashlib.sha256(p.cpu().numpy().tobytes()).hexdigest() == kk["weights_sha256"]
    assert hashlib.sha256(s.cpu().numpy().tobytes()).hexdigest() == kk["scales_sha256"]


def test_mxfp4_quantize_dequantize_golden(dev):
    g = np.load(os.path.join(GOLD, "golden.npz"))
    p, s = W.mxfp4_quantize(_bf16(g["mx_src_bits"], dev))
    np.testing.assert_array_equal(p.cpu().numpy(), g["mx_packed"])
    np.testing.assert_array_equal(s.cpu().numpy(), g["mx_scales"])
    d = W.mxfp4_dequantize(p, s, torch.float32).cpu().numpy()
    np.testing.assert_array_equal(d.view(np.uint32), g["mx_deq"].view(np.uint32))
    db = W.mxfp4_dequantize(p, s, torch.bfloat16)
    np.testing.assert_array_equal(_bits(db), F.f32_to_bf16_bits(g["mx_deq"]))


def test_mxfp4_random_large_and_extreme_scales(dev):
    rng = np.random.default_rng(11)
    w = rng.normal(0, 0.02, (512, 1024)).astype(np.float32)
    w[0] *= 1e30
    w[1] *= 1e-32
    w[2, :64] = 0
    w[3, ::7] = -0.0
    bits = F.f32_to_bf16_bits(w)
    p, s = W.mxfp4_quantize(_bf16(bits, dev))
    rp, rs = F.mxfp4_quantize_bf16(bits)
    np.testing.assert_array_equal(p.cpu().numpy(), rp)
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    # arbitrary bytes, every scale byte, dequant bit-exact (incl. 2^-127 and inf scales)
    pb = rng.integers(0, 256, (256, 512), dtype=np.uint8)
    sb = (np.arange(256 * 32, dtype=np.int64).reshape(256, 32) % 255).astype(np.uint8)  # 255 (inf) below
    d = W.mxfp4_dequantize(torch.from_numpy(pb).to(dev), torch.from_numpy(sb).to(dev), torch.float32).cpu().numpy()
    ref = F.mxfp4_dequantize(pb, sb)
    np.testing.assert_array_equal(d.view(np.uint32), ref.view(np.uint32))
    # scale byte 255 decodes to +inf: values are +-inf, and 0 * inf is NaN on both sides
    s255 = np.full((256, 32), 255, np.uint8)
    d = W.mxfp4_dequantize(torch.from_numpy(pb).to(dev), torch.from_numpy(s255).to(dev), torch.float32).cpu().numpy()
    with np.errstate(invalid="ignore"):
        np.testing.assert_array_equal(d, F.mxfp4_dequantize(pb, s255))


def test_affine4_golden(dev):
    g = np.load(os.path.join(GOLD, "golden.npz"))
    p, sc, bi = W.affine4_quantize(_bf16(g["af_src_bits"], dev), 64)
    np.testing.assert_array_equal(p.cpu().numpy().view(np.uint32), g["af_packed"])
    np.testing.assert_array_equal(_bits(sc), g["af_scales"])
    np.testing.assert_array_equal(_bits(bi), g["af_biases"])
    d = W.affine4_dequantize(p, sc, bi, 64, torch.float32).cpu().numpy()
    np.testing.assert_array_equal(d.view(np.uint32), g["af_deq"].view(np.uint32))


@pytest.mark.parametrize("fmt", range(6))
def test_kv_formats_golden(dev, fmt):
    g = np.load(os.path.join(GOLD, "golden.npz"))
    x = _bf16(g["kv_src_bits"], dev)
    p, s = W.kv_quantize(x, fmt)
    np.testing.assert_array_equal(p.cpu().numpy(), g[f"kv{fmt}_payload"])
    sc = s.cpu().numpy()
    exp = g[f"kv{fmt}_scales"]
    np.testing.assert_array_equal(sc.view(np.uint8), exp.view(np.uint8))
    d = W.kv_dequantize(p, s, fmt)
    np.testing.assert_array_equal(_bits(d), g[f"kv{fmt}_deq_bits"])


@pytest.mark.parametrize("fmt", range(6))
def test_kv_formats_random_vs_oracle(dev, fmt):
    rng = np.random.default_rng(100 + fmt)
    x = F.round_bf16((rng.standard_t(3, (301, 576)) * 3).astype(np.float32))
    x[7] = 0.0
    x[8, :32] = 1e-30
    bits = F.f32_to_bf16_bits(x)
    p, s = W.kv_quantize(_bf16(bits, dev), fmt)
    rp, rs = F.kv_quantize(x, fmt)
    np.testing.assert_array_equal(p.cpu().numpy(), rp)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint8), rs.view(np.uint8))
    idx = torch.tensor([[0, 300, 7], [-5, 1000, 150]], dtype=torch.int32, device=dev)
    gd = W.kv_gather_dequantize(p, s, idx, fmt)
    full = F.f32_to_bf16_bits(F.kv_dequantize(rp, rs, fmt, 576))
    rows = np.clip(idx.cpu().numpy(), 0, 300)
    np.testing.assert_array_equal(_bits(gd), full[rows])


def test_kv_bad_width_raises(dev):
    x = torch.zeros(4, 40, dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError):
        W.kv_quantize(x, "fp8_ue8m0")


@pytest.mark.gpu
@pytest.mark.parametrize("block,sf,fmt", [(64, 0, "fp8_f32_b64"), (32, 1, "fp8_ue8m0")])
def test_fp8_kv_named_entry_points(dev, block, sf, fmt):
    # wkv_fp8_quantize / wkv_fp8_dequantize give the bytes and values of the generic calls
    from whallm_b200 import _lib as C
    x = torch.randn(300, 576 if block == 64 else 512, device=dev).to(torch.bfloat16)
    p, s = W.kv_quantize(x, fmt)
    p2, s2 = torch.empty_like(p), torch.empty_like(s)
    rows, D = x.shape
    C.call("wkv_fp8_quantize", C.ptr(x), rows, D, block, sf, C.ptr(p2), C.ptr(s2), C.stream_of(x))
    out = torch.empty_like(x)
    C.call("wkv_fp8_dequantize", C.ptr(p2), C.ptr(s2), rows, D, block, sf, C.ptr(out), C.stream_of(x))
    torch.cuda.synchronize()
    assert torch.equal(p, p2) and torch.equal(s, s2)
    assert torch.equal(out, W.kv_dequantize(p, s, fmt))


def _all_finite_bf16_rows(D, order):
    b = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    b = b[((b.astype(np.uint32) >> 7) & 0xFF) != 0xFF]                  # drop inf / NaN
    if order == "shuffled":
        b = np.random.default_rng(5).permutation(b)
    else:
        b = b[np.argsort(np.abs(F.bf16_bits_to_f32(b)), kind="stable")]  # blocks of neighbouring magnitudes
    n = (len(b) // D) * D
    return b[:n].reshape(-1, D)


@pytest.mark.parametrize("fmt", [F.KV_FP8_F32_B64, F.KV_FP8_UE8M0_B32, F.KV_MXFP8_B32])
@pytest.mark.parametrize("order", ["shuffled", "sorted"])
def test_e4m3_kv_every_bf16_value_vs_oracle(dev, fmt, order):
    """Every finite bf16 value through the vectorised e4m3 row kernels: payload,
    scales and dequantized rows bit-exact against the oracle (sorted blocks
    put each scale over values of one magnitude, so every e4m3 binade,
    subnormals and rounding midpoints are reached)."""
    bits = _all_finite_bf16_rows(576 if fmt == F.KV_FP8_F32_B64 else 512, order)
    x = F.bf16_bits_to_f32(bits)
    p, s = W.kv_quantize(_bf16(bits, dev), fmt)
    rp, rs = F.kv_quantize(x, fmt)
    np.testing.assert_array_equal(p.cpu().numpy(), rp)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint8), rs.view(np.uint8))
    d = W.kv_dequantize(p, s, fmt)
    D = bits.shape[1]
    np.testing.assert_array_equal(_bits(d), F.f32_to_bf16_bits(F.kv_dequantize(rp, rs, fmt, D)))


def test_fp8_f32_scale_quotients_on_e4m3_midpoints(dev):
    """Blocks whose quotients v / s fall exactly on (and one bf16 step beside)
    e4m3 rounding midpoints, with scales that are not powers of two: the
    reciprocal product would round some of them the wrong way, the kernel's
    exact-division fallback must not."""
    mids = F.e4m3_to_f32(np.arange(1, 0x7E, dtype=np.uint8))
    mids = ((mids[:-1] + mids[1:]) / 2).astype(np.float32)            # midpoints between neighbouring codes
    rows = []
    for k in (3.0, 5.0, 7.0, 0.6, 1.7, 9.0, 11.0, 13.0):
        v = F.round_bf16((mids * np.float32(k)).astype(np.float32))
        v = np.concatenate([v, F.bf16_bits_to_f32(F.f32_to_bf16_bits(v) + 1), F.bf16_bits_to_f32(F.f32_to_bf16_bits(v) - 1)])
        for c0 in range(0, len(v), 63):
            blk = np.zeros(64, np.float32)
            chunk = v[c0:c0 + 63]
            blk[:len(chunk)] = chunk
            blk[63] = np.float32(448.0 * k)                              # amax, so s = float32(448 k / 448)
            rows.append(blk)
    flat = np.concatenate(rows)                                          # 64-value blocks, 9 per 576-row
    x = F.round_bf16(flat[: (flat.size // 576) * 576].reshape(-1, 576))
    bits = F.f32_to_bf16_bits(x)
    p, s = W.kv_quantize(_bf16(bits, dev), F.KV_FP8_F32_B64)
    rp, rs = F.kv_quantize(x, F.KV_FP8_F32_B64)
    np.testing.assert_array_equal(p.cpu().numpy(), rp)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint8), rs.view(np.uint8))


def test_fp8_dequantize_nan_codes_and_scales(dev):
    # NaN payload codes and non-finite scales take the scalar path: NaN is 0x7FC0 as in the oracle
    rng = np.random.default_rng(9)
    p = rng.integers(0, 256, (64, 576), dtype=np.uint8)
    p[0, :8] = 0x7F
    p[1, 8:16] = 0xFF
    s = rng.uniform(0.01, 2.0, (64, 9)).astype(np.float32)
    s[2, 0] = np.inf
    s[3, 1] = np.nan
    d = W.kv_dequantize(torch.from_numpy(p).to(dev), torch.from_numpy(s).to(dev), F.KV_FP8_F32_B64)
    with np.errstate(invalid="ignore"):
        ref = F.f32_to_bf16_bits(F.kv_dequantize(p, s, F.KV_FP8_F32_B64, 576))
    np.testing.assert_array_equal(_bits(d), ref)
