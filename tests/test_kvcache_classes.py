"""Reference-shaped KV caches on the device: V4.1 ``PackedRows``
(deepseek_v41/packed_cache.py:8-78) and the ``MXFP8PoolingCache`` quantized
storage (fp8_cache.py:59-240).

CPU: the constructors and ``restore`` reject what the reference rejects.

GPU: bytes written through ``PackedRows.write`` at slice and index-tensor
positions equal the oracle quantizer's, reads equal the oracle dequant, and
``grow``/``state``/``restore`` keep the bytes.  The pooling cache, driven
through updates that complete and leave open 64-row chunks, fetches exactly
the oracle's dequantized chunks plus the bf16 pending rows, gathers the same
rows, and scores queries against every cached row within the score kernel's
1e-2 max-relative tolerance (the D = 512 rows on the block-scaled tensor
cores, D = 128 through device dequant and one library GEMM).
"""
import numpy as np
import pytest
import torch

from oracle import formats as F
from oracle import moe as M
from whallm_b200.kvcache import MXFP8PoolingCache, PackedRows

KIND = {"fp8_ue8m0": F.KV_FP8_UE8M0_B32, "fp4_e4m3": F.KV_FP4_E4M3_B16, "fp4_ue8m0": F.KV_FP4_UE8M0_B32}


@pytest.mark.parametrize("kind,width", [("fp9", 64), ("fp4_e4m3", 24), ("fp8_ue8m0", 48)])
def test_packed_rows_rejects_bad_format(kind, width):
    with pytest.raises(ValueError, match="format or width"):
        PackedRows((1, 4, width), kind, device="cpu")


def test_packed_rows_restore_checks():
    r = PackedRows((1, 4, 64), "fp8_ue8m0", device="cpu")
    with pytest.raises(ValueError, match="does not match"):
        r.restore(dict(format="fp4_e4m3", payload=r.payload, scales=r.scales))
    with pytest.raises(ValueError, match="Invalid"):
        r.restore(dict(format="fp8_ue8m0", payload=r.payload[:, :2], scales=r.scales))
    bad = dict(format="fp8_ue8m0", payload=r.payload.to(torch.int16), scales=r.scales)
    with pytest.raises(ValueError, match="Invalid"):
        r.restore(bad)


def test_pooling_cache_state_arity():
    c = MXFP8PoolingCache(4, device="cpu")
    with pytest.raises(ValueError, match="3 or 5"):
        c.state = (None, None)


# --------------------------------------------------------------------------
# GPU
# --------------------------------------------------------------------------

def _np(t):
    return t.cpu().numpy()


def _f32(t):
    return t.float().cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["fp8_ue8m0", "fp4_e4m3", "fp4_ue8m0"])
def test_gpu_packed_rows_write_read(dev, kind):
    B, L, D = 2, 40, 512
    rows = PackedRows((B, L, D), kind)
    g = torch.Generator(device=dev).manual_seed(3)
    a = (torch.randn((B, 8, D), generator=g, device=dev) * 3).to(torch.bfloat16)
    slots = torch.tensor([1, 5, 6, 9, 20, 33, 34, 39], device=dev)
    rows.write((slice(None), slots), a)                          # index-tensor slots (cache.py:73)
    b = torch.randn((B, 4, D), generator=g, device=dev).to(torch.bfloat16)
    rows.write((slice(None), slice(10, 14)), b)                  # a slice
    f = KIND[kind]
    for val, idx in ((a, (slice(None), slots)), (b, (slice(None), slice(10, 14)))):
        p, s = F.kv_quantize(_f32(val).reshape(-1, D), f)
        np.testing.assert_array_equal(_np(rows.payload[idx]).reshape(p.shape), p)
        np.testing.assert_array_equal(_np(rows.scales[idx]).reshape(s.shape), s)
        want = F.kv_dequantize(p, s, f, D)
        got = rows[idx]
        assert got.dtype == torch.bfloat16 and tuple(got.shape) == (B, val.shape[1], D)
        np.testing.assert_array_equal(_f32(got).reshape(-1, D), F.round_bf16(want))
    big = rows.grow(64)
    assert tuple(big.payload.shape[:2]) == (B, 64)
    assert torch.equal(big.payload[:, :L], rows.payload) and torch.equal(big[:, :L], rows[:, :L])
    again = PackedRows((B, L, D), kind).restore(rows.state())
    assert torch.equal(again[:, :], rows[:, :])


def _oracle_rows(x, fmt, D):
    p, s = F.kv_quantize(x.reshape(-1, D), fmt)
    return p, s, F.round_bf16(F.kv_dequantize(p, s, fmt, D)).reshape(*x.shape[:-1], D)


@pytest.mark.gpu
@pytest.mark.parametrize("B,D", [(1, 512), (2, 512), (1, 128)])
def test_gpu_pooling_cache_vs_oracle(dev, B, D):
    g = torch.Generator(device=dev).manual_seed(B * 7 + D)
    cache = MXFP8PoolingCache(4)
    chunks = []
    for L in (30, 50, 70, 1, 200):         # 30 pending; 80 -> one chunk; 150 -> two; 151; 351 -> five
        px = torch.randn((B, L, D), generator=g, device=dev).to(torch.bfloat16)
        cache.update(px)
        chunks.append(px)
    allx = torch.cat(chunks, dim=1)
    n = 351 // 64 * 64
    assert cache.offset == 351 and cache.shape == (B, 351, D)
    done = _f32(allx[:, :n])
    _, _, deq8 = _oracle_rows(done, F.KV_MXFP8_B32, D)
    p4, s4, _ = _oracle_rows(done, F.KV_MXFP4_B32, D)
    # fetch: dequantized completed rows, then the bf16 pending rows
    got = cache.fetch(B, D, torch.bfloat16)
    np.testing.assert_array_equal(_f32(got[:, :n]), deq8)
    assert torch.equal(got[:, n:], allx[:, n:])
    # gather: rows by index, completed or pending
    idx = torch.randint(0, 351, (B, 3, 9), generator=g, device=dev, dtype=torch.int64)
    gath = cache.gather(idx)
    full = np.concatenate([deq8, _f32(allx[:, n:])], axis=1)
    want = np.stack([full[b][_np(idx[b])] for b in range(B)])
    np.testing.assert_array_equal(_f32(gath), want)
    # scores: every cached row; the indexer's copy is MXFP4
    q = torch.randn((B, 4, 2, D), generator=g, device=dev).to(torch.float32)
    s8 = cache.quantized_matmul(q)
    assert tuple(s8.shape) == (B, 4, 2, 351)
    qb = F.round_bf16(_f32(q).reshape(B, -1, D))
    ref8 = np.einsum("bqd,bld->bql", qb.astype(np.float64), full.astype(np.float64))
    assert M.max_rel_err(_f32(s8).reshape(B, -1, 351)[..., :n], ref8[..., :n]) < 1e-2
    ref_pend = np.einsum("bqd,bld->bql", _f32(q).reshape(B, -1, D).astype(np.float64),
                         _f32(allx[:, n:]).astype(np.float64))
    assert M.max_rel_err(_f32(s8).reshape(B, -1, 351)[..., n:], ref_pend) < 1e-4
    s4g = cache.index_matmul(q)
    deq4 = F.kv_dequantize(p4, s4, F.KV_MXFP4_B32, D).reshape(B, n, D)
    ref4 = np.einsum("bqd,bld->bql", qb.astype(np.float64), deq4.astype(np.float64))
    assert M.max_rel_err(_f32(s4g).reshape(B, -1, 351)[..., :n], ref4) < 1e-2
    # state: the dequantized history re-enters through update_and_fetch
    again = MXFP8PoolingCache(4)
    again.state = cache.state
    assert again.offset == 351 and torch.equal(again.fetch(B, D, torch.bfloat16), got)
    assert cache.make_mask(8, 100).shape == (8, 351)
