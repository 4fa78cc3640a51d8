"""Dense MXFP8 / MXFP4 linears on the block-scaled tensor path vs the oracle.

``MXFP8Linear`` mirrors the QuantizedLinear layers the reference installs over
native FP8 weights (deepseek_v41_ssd.py:232-261, 353-360): y = x @
dequant(W)^T with e4m3 W and one E8M0 scale per (row, 32 columns), the
scales expanded from 32 x 32 blocks.  Checked against the oracle's float64
product rounded to bf16 (1e-2 max-relative) for decode- and prefill-sized
token counts and weight heights that are not multiples of 128.  Decode-sized
calls that leave SMs idle split K across work items and add the f32 partial
sums in a fixed order: those results repeat bit for bit, and a workspace sized
for fewer splits gives the same answer through fewer splits.
"""
import numpy as np
import pytest
import torch

import whallm_b200 as W
from oracle import formats as F
from oracle import moe as M

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp4"])
@pytest.mark.parametrize("T,N,K", [(1, 512, 1024), (7, 1000, 7168), (3, 333, 512), (16, 5120, 5120),
                                   (200, 384, 2048)])
def test_mx_linear_vs_oracle(dev, fmt, T, N, K):
    g = torch.Generator(device=dev).manual_seed(T + N + K)
    w = (torch.randn((N, K), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn((T, K), generator=g, device=dev).to(torch.bfloat16)
    p, s = W.kv_quantize(w, fmt)
    y = W.mx_linear(x, p, s, fmt)
    f = {"mxfp8": F.KV_MXFP8_B32, "mxfp4": F.KV_MXFP4_B32}[fmt]
    ref = F.kv_scores(x.float().cpu().numpy()[None], p.cpu().numpy()[None], s.cpu().numpy()[None], f, K)[0]
    assert M.max_rel_err(y.float().cpu().numpy(), ref) < 1e-2
    assert torch.equal(W.mx_linear(x, p, s, fmt), y)          # split sums in a fixed order


def test_mx_linear_small_workspace_uses_fewer_splits(dev):
    from whallm_b200 import _lib as C
    T, N, K = 4, 2048, 4096
    g = torch.Generator(device=dev).manual_seed(5)
    w = (torch.randn((N, K), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn((T, K), generator=g, device=dev).to(torch.bfloat16)
    p, s = W.kv_quantize(w, "mxfp8")
    full = C.lib().wmx_linear_workspace_size(T, K, N)
    small = C.lib().wmx_linear_workspace_size(T, K, 1)          # room for the partials of one output column only
    assert small < full
    ws = torch.empty(small, dtype=torch.uint8, device=dev)
    y = torch.empty((T, N), dtype=torch.bfloat16, device=dev)
    C.call("wmx_linear", C.ptr(x), T, K, C.ptr(p), C.ptr(s), N, C.WKV_MXFP8_B32, C.ptr(y), C.ptr(ws), small,
           C.stream_of(x))
    ref = F.kv_scores(x.float().cpu().numpy()[None], p.cpu().numpy()[None], s.cpu().numpy()[None],
                      F.KV_MXFP8_B32, K)[0]
    assert M.max_rel_err(y.float().cpu().numpy(), ref) < 1e-2


def test_mxfp8_linear_from_native_fp8_blocks(dev):
    N, K = 70, 512
    g = torch.Generator(device=dev).manual_seed(1)
    wq = torch.randint(0, 256, (N, K), generator=g, device=dev, dtype=torch.uint8)
    wq[(wq & 0x7F) == 0x7F] = 0                      # no NaN codes
    blocks = torch.randint(110, 130, ((N + 31) // 32, K // 32), generator=g, device=dev, dtype=torch.uint8)
    lin = W.MXFP8Linear.from_native_fp8(wq, blocks)
    assert torch.equal(lin.scales[33], blocks[1]) and lin.scales.shape == (N, K // 32)
    x = torch.randn((3, K), generator=g, device=dev).to(torch.bfloat16)
    y = lin(x)
    ref = F.kv_scores(x.float().cpu().numpy()[None], wq.cpu().numpy()[None], lin.scales.cpu().numpy()[None],
                      F.KV_MXFP8_B32, K)[0]
    assert M.max_rel_err(y.float().cpu().numpy(), ref) < 1e-2
