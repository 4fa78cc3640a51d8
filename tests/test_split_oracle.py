"""The two-term e4m3 operand form (oracle restatement, CPU).

The block-scaled expert kernels feed bf16 activations to e4m3 tensor-core
inputs as x = 2^(s-127) * (hi + 2^-5 * lo).  This checks the restatement's
claims: exact for every element within 2^-14 of its 32-value block maximum,
at most 2^-22 of the block maximum off below that, block maxima scaled into
[128, 256), zeros and signed zeros preserved.
"""
import numpy as np

from oracle import formats as F


def _case(seed):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (48, 512)).astype(np.float32)
    x[1, :32] *= 1e-30                                  # tiny block
    x[2, :32] = 0.0                                     # zero block
    x[3, 7] = -0.0
    x[4, :32] *= np.logspace(-8, 8, 32)                 # wide dynamic range in one block
    x[5, 32:64] = 3e38                                  # near the bf16 maximum
    x[6, :] *= 1e4
    return F.f32_to_bf16_bits(x)


def test_split_is_exact_near_block_max():
    b = _case(1)
    hi, lo, sc = F.split_e4m3(b)
    x = F.bf16_bits_to_f32(b)
    y = F.join_e4m3(hi, lo, sc)
    blk = np.abs(x).reshape(x.shape[0], -1, 32).max(-1).repeat(32, 1)
    big = np.abs(x) >= blk * 2.0 ** -14
    np.testing.assert_array_equal(y[big], x[big])
    small = ~big & (blk > 0)
    assert (np.abs(y - x)[small] <= blk[small] * 2.0 ** -22).all()


def test_split_scales_and_signs():
    b = _case(2)
    hi, lo, sc = F.split_e4m3(b)
    x = F.bf16_bits_to_f32(b)
    blk = np.abs(x).reshape(x.shape[0], -1, 32).max(-1)
    s = sc.astype(np.int64) - 127
    nz = (blk > 0) & (s > -122)
    scaled = blk[nz] / np.exp2(s[nz].astype(np.float64))
    assert ((scaled >= 128) & (scaled < 256)).all()
    assert sc.min() >= 5                                 # the lo term's scale byte stays >= 0
    assert hi[3, 7] == 0x80 and lo[3, 7] == 0x00         # -0.0 keeps its sign in hi
    assert (hi[2, :32] == 0).all() and (lo[2, :32] == 0).all()
