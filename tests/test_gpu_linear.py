"""Dense MXFP8 / MXFP4 linears vs the oracle.

``MXFP8Linear`` mirrors the QuantizedLinear layers the reference installs over
native FP8 weights (deepseek_v41_ssd.py:232-261, 353-360): y = x @
dequant(W)^T with e4m3 W and one E8M0 scale per (row, 32 columns), the
scales expanded from 32 x 32 blocks.  Checked against the oracle's float64
product rounded to bf16 (1e-2 max-relative) for decode- and prefill-sized
token counts and weight heights that are not multiples of 128.  Decode-sized
calls that leave SMs idle split K across work items and add the f32 partial
sums in a fixed order: those results repeat bit for bit, and a workspace sized
for fewer splits gives the same answer through fewer splits.  One- and two-row
calls run on the CUDA-core weight stream (``linear_stream.cu``); they are
checked against the oracle and against the tensor path (``WM_LINEAR_PATH=tc``).
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


# ---- one- and two-row calls: the CUDA-core weight stream (linear_stream.cu)

def _linear_case(dev, fmt, T, N, K, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    w = (torch.randn((N, K), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn((T, K), generator=g, device=dev).to(torch.bfloat16)
    p, s = W.kv_quantize(w, fmt)
    f = {"mxfp8": F.KV_MXFP8_B32, "mxfp4": F.KV_MXFP4_B32}[fmt]
    ref = F.kv_scores(x.float().cpu().numpy()[None], p.cpu().numpy()[None], s.cpu().numpy()[None], f, K)[0]
    return x, p, s, ref


@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp4"])
@pytest.mark.parametrize("T", [1, 2])
@pytest.mark.parametrize("N,K", [(5120, 5120), (333, 512), (7, 7168), (1001, 7168), (7168, 1536), (130, 3072),
                                 (600, 18432), (4101, 1280)])
def test_stream_linear_vs_oracle_and_tensor_path(dev, monkeypatch, fmt, T, N, K):
    """Heights that are not multiples of the 4-row chunk, rows whose last 1024-value step is ragged (1536,
    3072, 1280), fewer chunks than SMs (a chunk's steps split into parts added in order), and two-row calls
    too wide to stage (18432 e4m3), which stay on the tensor path."""
    x, p, s, ref = _linear_case(dev, fmt, T, N, K, 11 * T + N + K)
    y = W.mx_linear(x, p, s, fmt)
    assert M.max_rel_err(y.float().cpu().numpy(), ref) < 1e-2
    assert torch.equal(W.mx_linear(x, p, s, fmt), y)                  # fixed order: repeats bit for bit
    monkeypatch.setenv("WM_LINEAR_PATH", "tc")
    y_tc = W.mx_linear(x, p, s, fmt)
    assert M.max_rel_err(y_tc.float().cpu().numpy(), ref) < 1e-2
    assert M.max_rel_err(y.float().cpu().numpy(), y_tc.float().cpu().numpy()) < 1e-2


@pytest.mark.parametrize("fmt", ["mxfp8", "mxfp4"])
def test_stream_linear_two_rows_equal_each_row_alone(dev, fmt):
    """Each (row, token) sum keeps its own chains, butterfly and segment order, so a two-row call gives
    every row's result bit for bit as a one-row call does."""
    x, p, s, _ = _linear_case(dev, fmt, 2, 3000, 3072, 7)
    y2 = W.mx_linear(x, p, s, fmt)
    for t in range(2):
        assert torch.equal(W.mx_linear(x[t:t + 1].contiguous(), p, s, fmt)[0], y2[t])


@pytest.mark.parametrize("T", [1, 2])
def test_stream_linear_every_e4m3_code(dev, T):
    """Random bytes over the whole e4m3 range (subnormals, both zeros, the largest finite values; no NaN
    codes) with scales far from 1: the stream widens each code to an exact f16 value."""
    N, K = 300, 2048
    g = torch.Generator(device=dev).manual_seed(3 + T)
    wq = torch.randint(0, 256, (N, K), generator=g, device=dev, dtype=torch.uint8)
    wq[(wq & 0x7F) == 0x7F] = 0
    sc = torch.randint(100, 150, (N, K // 32), generator=g, device=dev, dtype=torch.uint8)
    x = torch.randn((T, K), generator=g, device=dev).to(torch.bfloat16)
    y = W.mx_linear(x, wq, sc, "mxfp8")
    ref = F.kv_scores(x.float().cpu().numpy()[None], wq.cpu().numpy()[None], sc.cpu().numpy()[None],
                      F.KV_MXFP8_B32, K)[0]
    assert M.max_rel_err(y.float().cpu().numpy(), ref) < 1e-2
