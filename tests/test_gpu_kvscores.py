"""Scores against a quantized KV cache (MXFP8 chunks and the MXFP4 index copy)
on the block-scaled tensor cores vs the oracle.

MXFP8PoolingCache.quantized_matmul / index_matmul (fp8_cache.py:119-159) run
mx.quantized_matmul(query, packed K, transpose=True, group 32) over the
completed chunks.  The device path quantizes K with the library's bit-exact
kv_quantize, then computes the scores with e4m3 (MXFP8) or e2m1 (MXFP4) cache
rows as the MMA's A operand and the queries as two exact e4m3 terms; the
result must be within 1e-2 max-relative of the oracle's float64 product
rounded to bf16.  Cache lengths that are not a multiple of 128 and query
counts beyond one tile are covered.
"""
import numpy as np
import pytest
import torch

import whallm_b200 as W
from oracle import formats as F
from oracle import moe as M

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp4"])
@pytest.mark.parametrize("B,Lq,L,D", [(1, 1, 128, 512), (2, 5, 300, 512), (3, 40, 1000, 256), (1, 130, 640, 512)])
def test_kv_scores_vs_oracle(dev, fmt, B, Lq, L, D):
    g = torch.Generator(device=dev).manual_seed(B * 1000 + Lq * 10 + L)
    kv = torch.randn((B * L, D), generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn((B, Lq, D), generator=g, device=dev).to(torch.bfloat16)
    payload, scales = W.kv_quantize(kv, fmt)
    got = W.kv_scores(q, payload.view(B, L, -1), scales.view(B, L, -1), fmt)
    f = {"mxfp8": F.KV_MXFP8_B32, "mxfp4": F.KV_MXFP4_B32}[fmt]
    ref = F.kv_scores(q.float().cpu().numpy(), payload.view(B, L, -1).cpu().numpy(),
                      scales.view(B, L, -1).cpu().numpy(), f, D)
    assert M.max_rel_err(got.float().cpu().numpy(), ref) < 1e-2
