"""Qwen QSA affine-quantized KV cache (qwen_quantized_cache.py:6-57).

CPU: the 4/8-bit affine restatement agrees with the affine-4 one at 4 bits,
round-trips exactly on values it can represent, and the cache rejects what
the reference rejects (bits, width, persistence formats).

GPU: ``wkv_affine_append`` / ``wkv_affine_fetch`` equal the oracle bit for
bit (packed words, bf16 scales and biases, dequantized bf16), and a cache
driven through a prefill and decode steps that cross the 256-row growth
returns, at every step, exactly the oracle cache's history; a persisted and
restored cache continues identically.
"""
import numpy as np
import pytest
import torch

from oracle import formats as F
from whallm_b200 import _lib as C
from whallm_b200.kvcache import QSAQuantizedCache


def _bf16_bits(rng, shape, scale=1.0):
    return F.f32_to_bf16_bits((rng.standard_normal(shape) * scale).astype(np.float32))


def test_affine_restatement_at_4_bits_equals_affine4():
    x = F.bf16_bits_to_f32(_bf16_bits(np.random.default_rng(1), (16, 128)))
    for a, b in zip(F.affine_quantize(x, 32, 4), F.affine4_quantize(x, 32)):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("bits", [4, 8])
def test_affine_round_trip_on_representable_values(bits):
    # values scale*q + bias with q spanning 0..2^bits-1 in every group come back exactly
    rng = np.random.default_rng(bits)
    n = 2 ** bits - 1
    q = rng.integers(0, n + 1, (8, 64)).astype(np.float32)
    q[:, 0], q[:, 32] = 0, 0
    q[:, 1], q[:, 33] = n, n
    x = (q * np.float32(-0.125)).astype(np.float32)     # edge = min, exact, bias = min
    p, s, b = F.affine_quantize(x, 32, bits)
    np.testing.assert_array_equal(F.affine_dequantize(p, s, b, 32, bits), x)


@pytest.mark.parametrize("bits,dim", [(5, 128), (4, 100), (3, 64)])
def test_cache_rejects_bits_and_width(bits, dim):
    with pytest.raises(ValueError, match="4 or 8 bits"):
        QSAQuantizedCache(bits, dim)


def _saved(offset, width=16, groups=4, dtype=torch.bfloat16):
    part = (torch.zeros(1, 2, offset, width, dtype=torch.int32), torch.zeros(1, 2, offset, groups, dtype=dtype),
            torch.zeros(1, 2, offset, groups, dtype=dtype))
    return dict(bits=4, dimension=128, offset=offset, arrays=(part, part))


@pytest.mark.parametrize("saved,msg", [
    (dict(bits=8, dimension=128, offset=0, arrays=None), "format"),
    (dict(bits=4, dimension=128, offset=-1, arrays=None), "format"),
    (dict(bits=4, dimension=128, offset=3, arrays=None), "nonzero offset"),
    (dict(bits=4, dimension=128, offset=2, arrays=[1]), "arrays"),
    (_saved(3, width=8), "shape or dtype"),
    (_saved(3, dtype=torch.int8), "shape or dtype"),
])
def test_restore_rejects_bad_states(saved, msg):
    c = QSAQuantizedCache(4, 128)
    with pytest.raises(ValueError, match=msg):
        c.restore_persistence_state(saved)


def test_restore_adopts_a_valid_state():
    c = QSAQuantizedCache(4, 128)
    c.restore_persistence_state(_saved(5))
    assert c.offset == 5 and c.keys[0].shape == (1, 2, 5, 16)
    c.restore_persistence_state(dict(bits=4, dimension=128, offset=0, arrays=None))
    assert c.offset == 0 and c.keys is None


# --------------------------------------------------------------------------
# GPU
# --------------------------------------------------------------------------

def _t(bits_u16, dev):
    return torch.from_numpy(np.ascontiguousarray(bits_u16).view(np.int16)).to(dev).view(torch.bfloat16)


def _bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("n_seq,L,D,cap,off", [(2, 7, 128, 16, 3), (16, 1, 256, 300, 255), (4, 64, 64, 64, 0)])
def test_gpu_append_fetch_match_oracle(dev, bits, n_seq, L, D, cap, off):
    rng = np.random.default_rng(bits * 1000 + L)
    src = [_bf16_bits(rng, (n_seq, L, D), s) for s in (1.0, 3.0)]
    wd, g = D * bits // 32, D // 32
    caches = [(torch.zeros(n_seq, cap, wd, dtype=torch.int32, device=dev),
               torch.zeros(n_seq, cap, g, dtype=torch.bfloat16, device=dev),
               torch.zeros(n_seq, cap, g, dtype=torch.bfloat16, device=dev)) for _ in range(2)]
    k, v = _t(src[0], dev), _t(src[1], dev)
    (kq, ks, kb), (vq, vs, vb) = caches
    C.call("wkv_affine_append", C.ptr(k), C.ptr(v), n_seq, L, D, bits, C.ptr(kq), C.ptr(ks), C.ptr(kb), C.ptr(vq),
           C.ptr(vs), C.ptr(vb), cap, off, C.stream_of(k))
    outs = [torch.empty(n_seq, off + L, D, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    C.call("wkv_affine_fetch", C.ptr(kq), C.ptr(ks), C.ptr(kb), C.ptr(vq), C.ptr(vs), C.ptr(vb), n_seq, off + L, cap,
           D, bits, C.ptr(outs[0]), C.ptr(outs[1]), C.stream_of(k))
    torch.cuda.synchronize()
    for x, (q, s, b), out in zip(src, caches, outs):
        rq, rs, rb = F.affine_quantize(F.bf16_bits_to_f32(x.reshape(-1, D)), 32, bits)
        np.testing.assert_array_equal(q[:, off:off + L].cpu().numpy().view(np.uint32).reshape(-1, wd), rq)
        np.testing.assert_array_equal(_bits(s[:, off:off + L]).reshape(-1, g), rs)
        np.testing.assert_array_equal(_bits(b[:, off:off + L]).reshape(-1, g), rb)
        want = F.f32_to_bf16_bits(F.affine_dequantize(rq, rs, rb, 32, bits)).reshape(n_seq, L, D)
        np.testing.assert_array_equal(_bits(out[:, off:]), want)
        assert q[:, :off].eq(0).all() and q[:, off + L:].eq(0).all()    # other rows untouched


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 8])
def test_gpu_append_exact_ties(dev, bits):
    # groups with min -n/16 and max 0 get scale 1/16 and bias min, so
    # v = -(2k+1)/32 quantizes from exactly n - k - 1/2: every rounding tie
    # (and the values one bf16 step either side of it) must match the oracle
    n = 2 ** bits - 1
    rng = np.random.default_rng(bits)
    rows = []
    for _ in range(64):
        ks = rng.integers(0, min(n, 128), 32)     # 2k+1 < 256: exact in bf16
        v = -(2 * ks + 1) / 32.0
        v[0], v[1] = -n / 16.0, 0.0
        rows.append(v)
    x = np.asarray(rows, np.float32)
    nudged = F.bf16_bits_to_f32(F.f32_to_bf16_bits(x) + np.uint16(1))
    x = np.concatenate([x, np.where(np.arange(32) < 2, x, nudged)])
    xb = F.f32_to_bf16_bits(x).reshape(1, -1, 32)
    D = 32
    rows_n = xb.shape[1]
    caches = [(torch.zeros(1, rows_n, bits, dtype=torch.int32, device=dev),
               torch.zeros(1, rows_n, 1, dtype=torch.bfloat16, device=dev),
               torch.zeros(1, rows_n, 1, dtype=torch.bfloat16, device=dev))]
    k = _t(xb, dev)
    (kq, ks, kb), = caches
    C.call("wkv_affine_append", C.ptr(k), None, 1, rows_n, D, bits, C.ptr(kq), C.ptr(ks), C.ptr(kb), None, None,
           None, rows_n, 0, C.stream_of(k))
    torch.cuda.synchronize()
    rq, rs, rb = F.affine_quantize(F.bf16_bits_to_f32(xb.reshape(-1, D)), 32, bits)
    np.testing.assert_array_equal(kq.cpu().numpy().view(np.uint32).reshape(-1, bits), rq)
    np.testing.assert_array_equal(_bits(ks).reshape(-1, 1), rs)
    np.testing.assert_array_equal(_bits(kb).reshape(-1, 1), rb)


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 8])
def test_gpu_cache_steps_match_oracle_cache(dev, bits):
    B, H, D = 1, 4, 128
    rng = np.random.default_rng(7 + bits)
    ours, ref = QSAQuantizedCache(bits, D), F.QSACache(bits, D)
    for n in (300, 1, 1, 211, 1):      # grows 512 -> 768 rows on the way
        kb, vb = _bf16_bits(rng, (B, H, n, D)), _bf16_bits(rng, (B, H, n, D), 0.5)
        k, v = ours.update_and_fetch(_t(kb, dev), _t(vb, dev))
        rk, rv = ref.update_and_fetch(kb.reshape(B * H, n, D), vb.reshape(B * H, n, D))
        np.testing.assert_array_equal(_bits(k).reshape(B * H, -1, D), rk)
        np.testing.assert_array_equal(_bits(v).reshape(B * H, -1, D), rv)
    assert ours.offset == 514 and ours.keys[0].shape[2] == 768
    # persist, restore, continue: identical to continuing the original
    saved = ours.persistence_state()
    again = QSAQuantizedCache(bits, D)
    again.restore_persistence_state(saved)
    kb, vb = _bf16_bits(rng, (B, H, 2, D)), _bf16_bits(rng, (B, H, 2, D))
    a = ours.update_and_fetch(_t(kb, dev), _t(vb, dev))
    b = again.update_and_fetch(_t(kb, dev), _t(vb, dev))
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.gpu
def test_gpu_cache_reserved_capacity_never_moves(dev):
    c = QSAQuantizedCache(8, 64, capacity=1024)
    rng = np.random.default_rng(3)
    c.update_and_fetch(_t(_bf16_bits(rng, (1, 2, 10, 64)), dev), _t(_bf16_bits(rng, (1, 2, 10, 64)), dev))
    p = c.keys[0].data_ptr()
    for _ in range(3):
        c.update_and_fetch(_t(_bf16_bits(rng, (1, 2, 300, 64)), dev), _t(_bf16_bits(rng, (1, 2, 300, 64)), dev))
    assert c.keys[0].data_ptr() == p and c.offset == 910
    with pytest.raises(ValueError, match="width"):
        c.update_and_fetch(torch.zeros(1, 2, 1, 32, dtype=torch.bfloat16, device=dev),
                           torch.zeros(1, 2, 1, 32, dtype=torch.bfloat16, device=dev))
