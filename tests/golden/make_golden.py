"""Regenerate the committed golden fixtures in this folder.

1. ``mxfp4_kats.json`` -- the reference's own MXFP4 known-answer tests,
   extracted as text from
   ``Tests/DeepSeekRepackTests/DeepSeekRepackTests.swift:336-411``
   (testMXFP4MatchesMLXFixedVector, testMXFP4MatchesMLXBF16Rows,
   testMXFP4ConvertsOfficialFP8Blocks, testMXFP4FP8ConversionMatchesMLXFixedVector).
   Needs the reference checkout (pass its path as argv[1]); the GPU box never
   runs this.
2. ``golden.npz`` -- seeded small cases with the oracle's outputs (MXFP4
   quantize/dequantize, affine-4 dequant, every KV row format, the router for
   each score function), so device results are checked against frozen bytes
   as well as against the live oracle.

Usage:  python tests/golden/make_golden.py <reference-root>
"""
from __future__ import annotations

import json
import os
import re
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import formats as F  # noqa: E402
from oracle import router as R  # noqa: E402

SWIFT = "Tests/DeepSeekRepackTests/DeepSeekRepackTests.swift"


def _body(src: str, name: str) -> str:
    i = src.index(f"func {name}(")
    j = src.index("\n  func ", i + 1)
    return src[i:j]


def _ints(text: str):
    out = []
    for tok in re.findall(r"0x[0-9a-fA-F]+|\d+", text):
        out.append(int(tok, 16) if tok.startswith("0x") else int(tok))
    return out


def _repeat_list(text: str):
    """Parse `[a, b, ...] + Array(repeating: v, count: n)` into a list."""
    m = re.search(r"\[(.*?)\]\s*(\+\s*Array\(repeating:\s*([^,]+),\s*count:\s*(\d+)\))?", text, re.S)
    vals = [v.strip() for v in m.group(1).split(",") if v.strip()]
    if m.group(2):
        vals += [m.group(3).strip()] * int(m.group(4))
    return vals


def extract_kats(ref_root: str) -> dict:
    src = open(os.path.join(ref_root, SWIFT)).read()
    kats = {}
    b = _body(src, "testMXFP4MatchesMLXFixedVector")
    vals = [float(v) for v in _repeat_list(b[b.index("let values"):].split("=", 1)[1])]
    exp_w = _repeat_list(b[b.index("[UInt8](result.weights)"):].split(",", 1)[1])
    exp_s = _ints(b[b.index("[UInt8](result.scales)"):].split(",", 1)[1].split(")")[0])
    kats["fixed_vector"] = dict(values=vals, rows=1, cols=32,
                                weights=[int(v, 16) if v.startswith("0x") else int(v) for v in exp_w],
                                scales=exp_s)
    b = _body(src, "testMXFP4MatchesMLXBF16Rows")
    bits = _ints(b[b.index("let bits"):b.index("let source")].split("=", 1)[1])
    wpart = b[b.index("[UInt8](result.weights)"):b.index("[UInt8](result.scales)")]
    weights = _ints(wpart[wpart.index("[", 10):])
    scales = _ints(b[b.index("[UInt8](result.scales)"):].split(",", 1)[1].split(")")[0])
    kats["bf16_rows"] = dict(bits=bits, rows=2, cols=32, weights=weights, scales=scales)
    b = _body(src, "testMXFP4ConvertsOfficialFP8Blocks")
    first = _repeat_list(b[b.index("let firstRow"):].split("=", 1)[1])
    first = [int(v, 16) if v.startswith("0x") else int(v) for v in first]
    inv = _ints(b[b.index("inverseScales: Data("):].split(")")[0].split("(", 1)[1])
    exp_w = _repeat_list(b[b.index("result.weights.prefix(16)"):].split(",", 1)[1])
    exp_s = _ints(b[b.index("result.scales.prefix(4)"):].split(",", 1)[1].split(")")[0])
    kats["fp8_blocks"] = dict(first_row=first, rows=128, cols=128, inverse_scale_bytes=inv,
                              weights_prefix=[int(v, 16) if v.startswith("0x") else int(v) for v in exp_w],
                              scales_prefix=exp_s)
    b = _body(src, "testMXFP4FP8ConversionMatchesMLXFixedVector")
    mul, add = [int(v) for v in re.search(r"index \* (\d+) \+ (\d+)", b).groups()]
    inv = _ints(b[b.index("inverseScales: Data("):].split(")")[0].split("(", 1)[1])
    digests = re.findall(r'"([0-9a-f]{64})"', b)
    kats["fp8_sha256"] = dict(rows=128, cols=128, mul=mul, add=add, inverse_scale_bytes=inv,
                              weights_sha256=digests[0], scales_sha256=digests[1])
    kats["_source"] = f"{SWIFT} (testMXFP4* functions, lines 336-411)"
    return kats


def make_golden(path: str):
    rng = np.random.default_rng(20261201)
    g = {}
    # MXFP4 weights
    w = rng.normal(0, 0.02, (64, 256)).astype(np.float32)
    w[3, :32] = 0.0                      # an all-zero group
    w[5, 32:64] *= 1e-30                 # tiny values
    bits = F.f32_to_bf16_bits(w)
    p, s = F.mxfp4_quantize_bf16(bits)
    g["mx_src_bits"], g["mx_packed"], g["mx_scales"] = bits, p, s
    g["mx_deq"] = F.mxfp4_dequantize(p, s)
    # affine-4 dequant of a fixed quantization
    aw = F.round_bf16(rng.normal(0, 0.02, (32, 256)).astype(np.float32))
    ap, asc, abi = F.affine4_quantize(aw, 64)
    g["af_src_bits"], g["af_packed"], g["af_scales"], g["af_biases"] = F.f32_to_bf16_bits(aw), ap, asc, abi
    g["af_deq"] = F.affine4_dequantize(ap, asc, abi, 64)
    # KV formats on 576-wide rows
    x = F.round_bf16((rng.normal(0, 1, (37, 576)) * 2.3).astype(np.float32))
    x[4, :64] = 0.0
    g["kv_src_bits"] = F.f32_to_bf16_bits(x)
    for fmt in range(6):
        pl, sc = F.kv_quantize(x, fmt)
        g[f"kv{fmt}_payload"], g[f"kv{fmt}_scales"] = pl, sc
        g[f"kv{fmt}_deq_bits"] = F.f32_to_bf16_bits(F.kv_dequantize(pl, sc, fmt, 576))
    # router
    T, H, E, k = 13, 512, 64, 6
    xb = F.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32))
    wb = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    sb = (rng.normal(0, 0.3, E)).astype(np.float32)
    lb = (rng.normal(0, 0.5, E)).astype(np.float32)
    sg = F.f32_to_bf16_bits((rng.normal(0, 1, (H,)) / np.sqrt(H)).astype(np.float32))
    g["rt_x"], g["rt_w"], g["rt_sel_bias"], g["rt_logit_bias"], g["rt_shared_gate"] = xb, wb, sb, lb, sg
    cases = [(R.SCORE_SOFTMAX, None, lb, 0.0, 1.0, sg), (R.SCORE_SIGMOID, sb, None, 1e-20, 2.5, None),
             (R.SCORE_SQRTSOFTPLUS, sb, lb, 1e-20, 1.5, None), (R.SCORE_NONE, None, None, -1.0, 1.0, None)]
    for c, (fn, sel, lgb, eps, scale, shg) in enumerate(cases):
        logits, idx, wts, sh = R.route(xb, wb, k, fn, logit_bias=lgb, select_bias=sel, norm_eps=eps,
                                       route_scale=scale, wg_shared_bits=shg)
        g[f"rt{c}_logits"], g[f"rt{c}_idx"], g[f"rt{c}_w"] = logits, idx, wts
        if sh is not None:
            g[f"rt{c}_shared"] = sh
    np.savez_compressed(path, **g)


if __name__ == "__main__":
    if len(sys.argv) > 1:
        kats = extract_kats(sys.argv[1])
        with open(os.path.join(HERE, "mxfp4_kats.json"), "w") as f:
            json.dump(kats, f, indent=1)
    make_golden(os.path.join(HERE, "golden.npz"))
    print("wrote fixtures to", HERE)
