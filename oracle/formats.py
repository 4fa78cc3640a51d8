"""Bit-level number formats of the MoE / KV path, restated in numpy.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Every function cites the reference file:line it restates.  All arithmetic is
float32 with IEEE round-to-nearest-even, as the reference's MLX / Swift code
does; powers of two are applied exactly.
"""
from __future__ import annotations

import numpy as np

# e2m1 code -> value.  Code 8 ("negative zero") decodes to +0.0
# (deepseek_v41/dequant.py:27-30).
E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                 0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], np.float32)
E2M1_MAG = E2M1[:8]

FP8_MAX = np.float32(448.0)
FP4_MAX = np.float32(6.0)
FP8_MAX_INV = np.float32(1.0 / 448.0)  # fakequant.py:34
FP4_MAX_INV = np.float32(1.0 / 6.0)    # fakequant.py:35


# --------------------------------------------------------------------------
# bf16 <-> f32
# --------------------------------------------------------------------------

def bf16_bits_to_f32(bits) -> np.ndarray:
    """bf16 bit patterns (uint16) -> float32 (exact); MXFP4.swift:90-94."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)
    return b.view(np.float32)


def f32_to_bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even (MXFP4.swift:109-113).

    NaN inputs map to the quiet NaN 0x7FC0 (never produced on this path)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32).astype(np.uint64)
    r = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    r = r.astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), r)


def round_bf16(x) -> np.ndarray:
    """float32 -> nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# --------------------------------------------------------------------------
# E8M0 / ue8m0 scales
# --------------------------------------------------------------------------

def e8m0_to_f32(scale_u8) -> np.ndarray:
    """byte b -> 2**(b-127) exactly (dequant.py:33-36); b=255 -> inf."""
    e = np.asarray(scale_u8, dtype=np.int32) - 127
    with np.errstate(over="ignore"):
        return np.ldexp(np.float32(1.0), e).astype(np.float32)


def _log2_ceil_bits(x) -> np.ndarray:
    """ceil(log2 x) for positive normal float32 via IEEE bits (fakequant.py:47-52)."""
    bits = np.asarray(x, np.float32).view(np.uint32)
    exp = ((bits >> 23) & 0xFF).astype(np.int32) - 127
    man = (bits & 0x7FFFFF).astype(np.int32)
    return exp + (man != 0).astype(np.int32)


def _pow2(e) -> np.ndarray:
    """2**e for integer e via IEEE bits (fakequant.py:55-57)."""
    return ((np.asarray(e, np.int64) + 127) << 23).astype(np.uint32).view(np.float32)


def ue8m0_scale(amax, max_inv) -> np.ndarray:
    """fast_round_scale: 2**ceil(log2(amax * (1/max))) (fakequant.py:60-62)."""
    prod = (np.asarray(amax, np.float32) * np.float32(max_inv)).astype(np.float32)
    return _pow2(_log2_ceil_bits(prod))


# --------------------------------------------------------------------------
# e4m3fn (FP8) encode / decode
# --------------------------------------------------------------------------

def e4m3_to_f32(code) -> np.ndarray:
    """Decode e4m3fn bytes (MXFP4.swift:96-107): subnormals m*2^-9, 0x7F/0xFF NaN."""
    c = np.asarray(code, np.uint8).astype(np.int32)
    sign = np.where(c & 0x80, np.float32(-1.0), np.float32(1.0))
    e = (c >> 3) & 0xF
    m = c & 7
    sub = m.astype(np.float32) * np.float32(2.0 ** -9)
    nrm = np.ldexp((np.float32(1.0) + m.astype(np.float32) / np.float32(8.0)), e - 7).astype(np.float32)
    v = np.where(e == 0, sub, nrm).astype(np.float32) * sign
    return np.where((e == 15) & (m == 7), np.float32(np.nan), v).astype(np.float32)


def f32_to_e4m3(x) -> np.ndarray:
    """float32 -> e4m3fn byte, round to nearest even, saturating at +-448.

    This is ``mx.to_fp8`` as used after ``clip(., -448, 448)``
    (packed_cache.py:38, fakequant.py:88); callers clip first, so the
    saturation is never exercised on the path.  Finite inputs only."""
    x = np.asarray(x, np.float32)
    sign = (x.view(np.uint32) >> 31).astype(np.uint8) << 7
    a = np.minimum(np.abs(x), FP8_MAX).astype(np.float64)  # exact copy of the f32 value
    # quantum for |a|: normals [2^-6, 448]: 2^(floor(log2 a) - 3); subnormals: 2^-9.
    # floor(log2 a) comes from frexp, exact at powers of two.
    _, e2 = np.frexp(np.where(a > 0, a, 1.0))
    ex = np.maximum(e2 - 1, -6).astype(np.float64)
    q = np.ldexp(1.0, (ex - 3).astype(np.int64))
    n = np.rint(a / q)               # a/q exact (power-of-two divide); rint = half-even
    v = n * q                        # rounded magnitude, exactly representable
    # re-derive exponent/mantissa from the rounded value
    v = np.minimum(v, 448.0)
    out = np.zeros(x.shape, np.uint8)
    nz = v > 0
    mm, ee = np.frexp(np.where(nz, v, 1.0))   # v = mm * 2^ee, mm in [0.5, 1)
    e_unb = ee - 1                            # v = (2mm) * 2^e_unb
    is_norm = nz & (e_unb >= -6)
    mant_n = np.rint((2 * mm - 1.0) * 8).astype(np.int64)
    code_n = ((e_unb + 7) << 3) | mant_n
    code_s = np.rint(v / 2.0 ** -9).astype(np.int64)
    code = np.where(is_norm, code_n, np.where(nz, code_s, 0))
    out[...] = code.astype(np.uint8)
    return (out | sign).astype(np.uint8)


# --------------------------------------------------------------------------
# e2m1 (FP4)
# --------------------------------------------------------------------------

def e2m1_code(v) -> np.ndarray:
    """Swift ``fp4Code`` (MXFP4.swift:115-131): nearest e2m1 magnitude, ties to
    the even code index, saturating at 6; the sign bit follows the float's
    sign bit (so -0.0 and small negatives give code 8)."""
    v = np.asarray(v, np.float32)
    neg = (v.view(np.uint32) >> 31).astype(np.uint8)
    mag = np.minimum(np.abs(v), FP4_MAX)
    idx = ((mag > 0.25).astype(np.uint8) + (mag >= 0.75) + (mag > 1.25) + (mag >= 1.75)
           + (mag > 2.5) + (mag >= 3.5) + (mag > 5.0)).astype(np.uint8)
    return (idx | (neg << 3)).astype(np.uint8)


def e2m1_code_loop(value: float) -> int:
    """Literal scalar restatement of MXFP4.swift:115-131 (used to pin e2m1_code)."""
    v = np.float32(value)
    negative = bool(np.signbit(v))
    magnitude = min(abs(v), np.float32(6))
    selected, distance = 0, np.float32(np.inf)
    for index, cand in enumerate(E2M1_MAG):
        d = np.float32(abs(magnitude - cand))
        if d < distance or (d == distance and index % 2 == 0):
            selected, distance = index, d
    return selected | (8 if negative else 0)


def e2m1_round(v) -> np.ndarray:
    """fakequant._e2m1_round (fakequant.py:65-73): ties-to-even on the grid."""
    v = np.asarray(v, np.float32)
    mag = np.abs(v)
    idx = np.zeros(mag.shape, np.int32)
    for t in (0.25, 1.25, 2.5, 5.0):
        idx += (mag > np.float32(t))
    for t in (0.75, 1.75, 3.5):
        idx += (mag >= np.float32(t))
    return (np.sign(v) * E2M1_MAG[idx]).astype(np.float32)


def pack_nibbles(codes) -> np.ndarray:
    """[..., 2n] codes -> [..., n] bytes, low nibble = even index (dequant.py:53-60)."""
    c = np.asarray(codes, np.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def unpack_nibbles(packed) -> np.ndarray:
    p = np.asarray(packed, np.uint8)
    out = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), np.uint8)
    out[..., 0::2] = p & 0xF
    out[..., 1::2] = p >> 4
    return out


# --------------------------------------------------------------------------
# MXFP4 weights (Swift repacker quantizer, MLX-compatible layout)
# --------------------------------------------------------------------------

def _float_exponent(a) -> np.ndarray:
    """Swift ``Float.exponent`` for positive finite a: floor(log2 a), subnormals included."""
    _, e = np.frexp(np.asarray(a, np.float32))
    return (e - 1).astype(np.int32)


def mxfp4_quantize_values(vals: np.ndarray):
    """Quantize float32 [rows, cols] (cols % 32 == 0) with the Swift MXFP4 rule.

    MXFP4.swift:19-37: per 32-value group, amax == 0 leaves scale 0 and codes 0;
    otherwise e = clamp(exponent(amax) - 2, -127, 128), scale byte e + 127,
    values scaled by 2^-e and rounded with fp4Code.
    Returns (packed uint8 [rows, cols/2], scales uint8 [rows, cols/32])."""
    v = np.ascontiguousarray(vals, np.float32)
    rows, cols = v.shape
    if cols % 32:
        raise ValueError("MXFP4 source must contain complete 32-value groups")
    g = v.reshape(rows, cols // 32, 32)
    amax = np.max(np.abs(g), axis=-1)
    zero = amax == 0
    e = np.clip(_float_exponent(np.where(zero, 1.0, amax)) - 2, -127, 128)
    scales = np.where(zero, 0, e + 127).astype(np.uint8)
    factor = np.ldexp(np.float32(1.0), -e).astype(np.float32)
    scaled = (g * factor[..., None]).astype(np.float32)
    codes = e2m1_code(scaled)
    codes[zero] = 0
    return pack_nibbles(codes.reshape(rows, cols)), scales


def mxfp4_quantize_bf16(src_bits) -> tuple[np.ndarray, np.ndarray]:
    """MXFP4.quantizeBF16 (MXFP4.swift:4-40) on bf16 bit patterns [rows, cols]."""
    return mxfp4_quantize_values(bf16_bits_to_f32(src_bits))


def mxfp4_quantize_fp8(src_u8, inverse_scales_bf16_bits, rows: int, cols: int):
    """MXFP4.quantizeFP8 (MXFP4.swift:42-88): 128x128-block e4m3 checkpoint
    weights times their bf16 inverse scale, rounded to bf16, then the MXFP4 rule."""
    if rows % 128 or cols % 128:
        raise ValueError("MXFP4 FP8 source must contain complete 128 by 128 scale blocks")
    src = np.asarray(src_u8, np.uint8).reshape(rows, cols)
    inv = bf16_bits_to_f32(np.asarray(inverse_scales_bf16_bits, np.uint16)).reshape(rows // 128, cols // 128)
    s = np.repeat(np.repeat(inv, 128, axis=0), 128, axis=1)
    vals = round_bf16((e4m3_to_f32(src) * s).astype(np.float32))
    return mxfp4_quantize_values(vals)


def mxfp4_dequantize(packed, scales) -> np.ndarray:
    """dequant_fp4 (dequant.py:63-66): e2m1[code] * 2^(s-127), float32 [rows, cols]."""
    codes = unpack_nibbles(packed)
    w = E2M1[codes]
    s = e8m0_to_f32(scales)
    rows, cols = w.shape[-2], w.shape[-1]
    return (w.reshape(*w.shape[:-1], cols // 32, 32) * s[..., None]).reshape(w.shape).astype(np.float32)


# --------------------------------------------------------------------------
# MLX-style affine 4-bit, group 64 (tiny config)
# --------------------------------------------------------------------------

def affine4_quantize(w_bf16_values: np.ndarray, group: int = 64):
    """Affine 4-bit quantizer following MLX's published affine scheme.

    PARITY UNPINNED: the reference only round-trips MLX against itself
    (runtime/tests/test_qwen_quantized_cache.py:10-16), so no vector pins the
    quantizer.  This restatement fixes the rule used for the synthetic weights:
    per group, the endpoint with the larger magnitude is made exact
    (edge = w_min if |w_min| > |w_max| else w_max), scale = +-(max-min)/15
    (>= 1e-7 in magnitude) nudged so edge/scale is an integer q0, bias = edge
    (0 when q0 == 0), q = clip(rint((w - bias)/scale), 0, 15); scales and biases
    are stored as bf16.  Packing: 8 nibbles per uint32, element 0 in the low
    nibble (engram.py:207-221 shapes).  The dequant of (q, scale, bias) is the
    pinned part: w = float32(scale) * q + float32(bias)."""
    w = np.ascontiguousarray(w_bf16_values, np.float32)
    rows, cols = w.shape
    if cols % group or group % 8:
        raise ValueError("affine4 needs cols % group == 0")
    g = w.reshape(rows, cols // group, group)
    w_max = g.max(-1)
    w_min = g.min(-1)
    mask = np.abs(w_min) > np.abs(w_max)
    scale = np.maximum((w_max - w_min) / np.float32(15.0), np.float32(1e-7)).astype(np.float32)
    scale = np.where(mask, scale, -scale).astype(np.float32)
    edge = np.where(mask, w_min, w_max).astype(np.float32)
    q0 = np.rint(edge / scale).astype(np.float32)
    scale = np.where(q0 != 0, edge / np.where(q0 != 0, q0, 1), scale).astype(np.float32)
    bias = np.where(q0 == 0, np.float32(0), edge).astype(np.float32)
    q = np.clip(np.rint((g - bias[..., None]) / scale[..., None]), 0, 15).astype(np.uint32)
    q = q.reshape(rows, cols // 8, 8)
    packed = np.zeros((rows, cols // 8), np.uint32)
    for i in range(8):
        packed |= q[..., i] << np.uint32(4 * i)
    return packed, f32_to_bf16_bits(scale), f32_to_bf16_bits(bias)


def affine4_dequantize(packed_u32, scales_bf16_bits, biases_bf16_bits, group: int = 64) -> np.ndarray:
    """w = scale * q + bias in float32 (scale*q is exact), float32 [rows, cols]."""
    p = np.asarray(packed_u32, np.uint32)
    rows, words = p.shape
    q = np.empty((rows, words, 8), np.float32)
    for i in range(8):
        q[..., i] = ((p >> np.uint32(4 * i)) & 0xF).astype(np.float32)
    q = q.reshape(rows, words * 8)
    s = bf16_bits_to_f32(scales_bf16_bits)
    b = bf16_bits_to_f32(biases_bf16_bits)
    qg = q.reshape(rows, -1, group)
    return (qg * s[..., None] + b[..., None]).reshape(rows, -1).astype(np.float32)


def affine_quantize(w_bf16_values: np.ndarray, group: int = 32, bits: int = 4):
    """The affine scheme of ``affine4_quantize`` for 4 or 8 bits
    (2**bits - 1 steps per group); 32/bits values per uint32, element 0 in the
    lowest bits.  Same parity status as ``affine4_quantize``: the quantizer
    is unpinned, the dequant w = scale * q + bias is the pinned part."""
    if bits not in (4, 8):
        raise ValueError("affine bits must be 4 or 8")
    w = np.ascontiguousarray(w_bf16_values, np.float32)
    rows, cols = w.shape
    if cols % group or group % 32:
        raise ValueError("affine needs cols % group == 0")
    nbins = np.float32(2 ** bits - 1)
    g = w.reshape(rows, cols // group, group)
    w_max = g.max(-1)
    w_min = g.min(-1)
    mask = np.abs(w_min) > np.abs(w_max)
    scale = np.maximum((w_max - w_min) / nbins, np.float32(1e-7)).astype(np.float32)
    scale = np.where(mask, scale, -scale).astype(np.float32)
    edge = np.where(mask, w_min, w_max).astype(np.float32)
    q0 = np.rint(edge / scale).astype(np.float32)
    scale = np.where(q0 != 0, edge / np.where(q0 != 0, q0, 1), scale).astype(np.float32)
    bias = np.where(q0 == 0, np.float32(0), edge).astype(np.float32)
    q = np.clip(np.rint((g - bias[..., None]) / scale[..., None]), 0, nbins).astype(np.uint32)
    per = 32 // bits
    q = q.reshape(rows, cols // per, per)
    packed = np.zeros((rows, cols // per), np.uint32)
    for i in range(per):
        packed |= q[..., i] << np.uint32(bits * i)
    return packed, f32_to_bf16_bits(scale), f32_to_bf16_bits(bias)


def affine_dequantize(packed_u32, scales_bf16_bits, biases_bf16_bits, group: int = 32, bits: int = 4) -> np.ndarray:
    """w = float32(scale) * q + float32(bias), float32 [rows, cols]."""
    p = np.asarray(packed_u32, np.uint32)
    rows, words = p.shape
    per = 32 // bits
    mask = np.uint32(2 ** bits - 1)
    q = np.empty((rows, words, per), np.float32)
    for i in range(per):
        q[..., i] = ((p >> np.uint32(bits * i)) & mask).astype(np.float32)
    q = q.reshape(rows, -1, group)
    s = bf16_bits_to_f32(scales_bf16_bits)
    b = bf16_bits_to_f32(biases_bf16_bits)
    return (q * s[..., None] + b[..., None]).reshape(rows, -1).astype(np.float32)


class QSACache:
    """The Qwen QSA quantized KV cache (qwen_quantized_cache.py:6-20) on
    mlx-lm's QuantizedKVCache: every update quantizes the new keys and values
    (group 32, ``bits``), appends them, and returns the whole history
    dequantized (bf16 bit patterns [n_seq, offset, D]).  Storage growth is not
    modelled: it does not change the values."""

    def __init__(self, bits: int, dimension: int):
        if bits not in (4, 8) or dimension % 32:
            raise ValueError("QSA quantized cache requires 4 or 8 bits and a width divisible by 32")
        self.bits, self.dimension = bits, dimension
        self.parts = None      # [(q, s, b) for keys, values], rows of all sequences as [n_seq, offset, width]

    def update_and_fetch(self, keys_bf16_bits, values_bf16_bits):
        out = []
        new_parts = []
        for i, x in enumerate((keys_bf16_bits, values_bf16_bits)):
            n_seq, L, D = x.shape
            if D != self.dimension:
                raise ValueError("QSA cache width does not match")
            q, s, b = affine_quantize(bf16_bits_to_f32(x.reshape(-1, D)), 32, self.bits)
            q, s, b = q.reshape(n_seq, L, -1), s.reshape(n_seq, L, -1), b.reshape(n_seq, L, -1)
            if self.parts is not None:
                pq, ps, pb = self.parts[i]
                q, s, b = (np.concatenate([pq, q], 1), np.concatenate([ps, s], 1), np.concatenate([pb, b], 1))
            new_parts.append((q, s, b))
            n, T, _ = q.shape
            w = affine_dequantize(q.reshape(n * T, -1), s.reshape(n * T, -1), b.reshape(n * T, -1), 32, self.bits)
            out.append(f32_to_bf16_bits(w).reshape(n, T, D))
        self.parts = new_parts
        return tuple(out)


# --------------------------------------------------------------------------
# KV-cache row formats
# --------------------------------------------------------------------------

KV_FP8_F32_B64 = 0    # fp32 scale = amax/448 per 64 values
KV_FP8_UE8M0_B32 = 1  # PackedRows 'fp8_ue8m0' (packed_cache.py:24-45)
KV_FP4_E4M3_B16 = 2   # PackedRows 'fp4_e4m3'
KV_FP4_UE8M0_B32 = 3  # PackedRows 'fp4_ue8m0'
KV_MXFP8_B32 = 4      # MXFP8 (e4m3 + E8M0 per 32), OCP MX v1.0 conversion rule
KV_MXFP4_B32 = 5      # MXFP4 index copy (e2m1 + E8M0 per 32), Swift/MLX rule

KV_BLOCK = {0: 64, 1: 32, 2: 16, 3: 32, 4: 32, 5: 32}
KV_BITS = {0: 8, 1: 8, 2: 4, 3: 4, 4: 8, 5: 4}
KV_SCALE_BYTES = {0: 4, 1: 1, 2: 1, 3: 1, 4: 1, 5: 1}


def kv_quantize(x_f32: np.ndarray, fmt: int):
    """Quantize rows [..., D] (values already bf16-representable) into
    (payload uint8 [..., D*bits/8], scales [..., D/block]).

    fmt 1-3 restate PackedRows.write (packed_cache.py:24-45):
      ue8m0:  s = 2^ceil(log2(max(amax, floor) * (1/max))), byte = exponent field,
              fp8 payload = to_fp8(clip(x/s, +-448)); fp4 payload = e2m1 code of
              _e2m1_round(clip(x/s, +-6)) with code = #(|r| > LUT) | (r<0)<<3.
      e4m3 scale (fp4_e4m3): s = from_fp8(to_fp8(max(amax, 6*2^-9)/6)).
    fmt 0 (BASELINE): s = amax/448 in fp32 (amax == 0 -> s = 0, payload 0),
      payload = to_fp8(clip(x/s, +-448)); scales stored as float32.
    fmt 4 (MXFP8: mx.quantize(mode="mxfp8"), fp8_cache.py:112): the OCP
      Microscaling Formats (MX) Specification v1.0 conversion of a 32-value
      block to MXFP8 E4M3 (section 6.3; E8M0 scale section 5.4; E4M3 element
      section 5.3): shared exponent X = floor(log2 max|V|) - emax_elem with
      emax_elem = 8 for E4M3 (largest normal 1.75 * 2^8 = 448), stored as the
      E8M0 byte X + 127 and clamped to the byte's finite range [-127, 127];
      elements P_i = V_i / 2^X rounded to nearest even in E4M3 and clamped to
      +-448 (E4M3 has no infinity, overflows saturate); a block of zeros
      (log2 0 undefined) stores scale byte 0 and zero elements.  The same rule
      with emax_elem = 2 (E2M1) is what the Swift MXFP4 quantizer implements
      (MXFP4.swift:19-37, pinned by its known-answer tests).
    fmt 5 (MXFP4 index copy): the Swift MXFP4 rule (mxfp4_quantize_values)."""
    x = np.ascontiguousarray(x_f32, np.float32)
    D = x.shape[-1]
    blk = KV_BLOCK[fmt]
    if D % blk:
        raise ValueError("Invalid packed cache format or width")
    lead = x.shape[:-1]
    if fmt == KV_MXFP4_B32:
        p, s = mxfp4_quantize_values(x.reshape(-1, D))
        return p.reshape(*lead, D // 2), s.reshape(*lead, D // 32)
    b = x.reshape(*lead, D // blk, blk)
    amax = np.max(np.abs(b), axis=-1, keepdims=True)
    if fmt == KV_FP8_F32_B64:
        scale = (amax / FP8_MAX).astype(np.float32)
        safe = np.where(scale > 0, scale, np.float32(1.0))
        q = np.where(scale > 0, np.clip(b / safe, -FP8_MAX, FP8_MAX), np.float32(0)).astype(np.float32)
        payload = f32_to_e4m3(q).reshape(*lead, D)
        return payload, scale[..., 0].astype(np.float32)
    if fmt == KV_MXFP8_B32:
        zero = amax == 0
        e = np.clip(_float_exponent(np.where(zero, 1.0, amax)) - 8, -127, 127)
        f = np.ldexp(np.float32(1.0), -e).astype(np.float32)
        q = np.clip((b * f).astype(np.float32), -FP8_MAX, FP8_MAX)
        q = np.where(zero, np.float32(0), q)
        payload = f32_to_e4m3(q).reshape(*lead, D)
        return payload, np.where(zero, 0, e + 127)[..., 0].astype(np.uint8)
    if fmt == KV_FP4_E4M3_B16:
        enc = f32_to_e4m3((np.maximum(amax, np.float32(6.0 * 2.0 ** -9)) / FP4_MAX).astype(np.float32))
        scale = e4m3_to_f32(enc)
    else:
        bits8 = fmt == KV_FP8_UE8M0_B32
        floor, inv = ((np.float32(1e-4), FP8_MAX_INV) if bits8 else (np.float32(6.0 * 2.0 ** -126), FP4_MAX_INV))
        scale = ue8m0_scale(np.maximum(amax, floor), inv)
        enc = ((scale.view(np.uint32) >> 23) & 255).astype(np.uint8)
    scaled = (b / scale).astype(np.float32)
    if fmt == KV_FP8_UE8M0_B32:
        payload = f32_to_e4m3(np.clip(scaled, -FP8_MAX, FP8_MAX)).reshape(*lead, D)
    else:
        r = e2m1_round(np.clip(scaled, -FP4_MAX, FP4_MAX))
        code = np.sum(np.abs(r)[..., None] > E2M1_MAG, axis=-1).astype(np.uint8)
        code = (code | ((r < 0).astype(np.uint8) << 3)).reshape(*lead, D)
        payload = pack_nibbles(code)
    return payload, enc[..., 0]


def kv_dequantize(payload, scales, fmt: int, D: int) -> np.ndarray:
    """PackedRows.__getitem__ (packed_cache.py:47-59) and the fmt-0/4/5 analogues:
    value = decode(payload) * scale, float32 [..., D] (callers round to bf16)."""
    blk = KV_BLOCK[fmt]
    p = np.asarray(payload, np.uint8)
    lead = p.shape[:-1]
    if KV_BITS[fmt] == 8:
        v = e4m3_to_f32(p)
    else:
        codes = unpack_nibbles(p)
        if fmt == KV_MXFP4_B32:
            v = E2M1[codes]
        else:
            v = (E2M1_MAG[(codes & 7).astype(np.int32)] * np.where(codes & 8, np.float32(-1.0), np.float32(1.0))).astype(np.float32)
    if fmt == KV_FP8_F32_B64:
        s = np.asarray(scales, np.float32)
    elif fmt == KV_FP4_E4M3_B16:
        s = e4m3_to_f32(scales)
    elif fmt in (KV_MXFP8_B32, KV_MXFP4_B32):
        s = e8m0_to_f32(scales)
    else:
        s = (np.asarray(scales, np.uint8).astype(np.uint32) << 23).view(np.float32)
    out = v.reshape(*lead, D // blk, blk) * s[..., None]
    return out.reshape(*lead, D).astype(np.float32)


def fake_quant(x_f32: np.ndarray, kind: str) -> np.ndarray:
    """fakequant.fake_quant_* (fakequant.py:83-119), float32 result.

    kind: 'fp8_ue8m0' (block 32), 'fp4_ue8m0' (block 32), 'fp4_e4m3' (block 16)."""
    x = np.asarray(x_f32, np.float32)
    D = x.shape[-1]
    if kind == "fp8_ue8m0":
        blk = 32
    elif kind == "fp4_ue8m0":
        blk = 32
    elif kind == "fp4_e4m3":
        blk = 16
    else:
        raise ValueError(kind)
    if D % blk:
        raise ValueError(f"last dim {D} not divisible by block {blk}")
    b = x.reshape(*x.shape[:-1], D // blk, blk)
    if kind == "fp8_ue8m0":
        amax = np.maximum(np.max(np.abs(b), -1, keepdims=True), np.float32(1e-4))
        s = ue8m0_scale(amax, FP8_MAX_INV)
        q = e4m3_to_f32(f32_to_e4m3(np.clip(b / s, -FP8_MAX, FP8_MAX))) * s
    elif kind == "fp4_ue8m0":
        amax = np.maximum(np.max(np.abs(b), -1, keepdims=True), np.float32(6.0 * 2.0 ** -126))
        s = ue8m0_scale(amax, FP4_MAX_INV)
        q = e2m1_round(np.clip(b / s, -FP4_MAX, FP4_MAX)) * s
    else:
        amax = np.maximum(np.max(np.abs(b), -1, keepdims=True), np.float32(6.0 * 2.0 ** -9))
        s = e4m3_to_f32(f32_to_e4m3((amax / FP4_MAX).astype(np.float32)))
        q = e2m1_round(np.clip(b / s, -FP4_MAX, FP4_MAX)) * s
    return q.reshape(x.shape).astype(np.float32)


PACKED_KIND_TO_FMT = {"fp8_ue8m0": KV_FP8_UE8M0_B32, "fp4_e4m3": KV_FP4_E4M3_B16, "fp4_ue8m0": KV_FP4_UE8M0_B32}


# --------------------------------------------------------------------------
# two-term e4m3 operand form (block-scaled expert kernels)
# --------------------------------------------------------------------------

LO_SHIFT = 5


def split_e4m3(x_bits):
    """bf16 bits [rows, cols] -> (hi, lo, scales) u8, the token operand of the
    block-scaled expert path (not a reference format: the decomposition that
    lets MXFP4 weights meet bf16 activations on e4m3 tensor-core inputs).

    Per 32 values: sh = max(exponent(block max) - 7, -122) so that
    block max / 2^sh lies in [128, 256); hi = e4m3(x / 2^sh) and
    lo = e4m3((x / 2^sh - hi) * 2^5), round to nearest even; scale = sh + 127."""
    b = np.asarray(x_bits, np.uint16)
    rows, cols = b.shape
    x = bf16_bits_to_f32(b).reshape(rows, cols // 32, 32)
    amax = (x.view(np.uint32) & np.uint32(0x7FFFFFFF)).max(axis=-1)
    ebits = np.minimum(amax >> np.uint32(23), np.uint32(255)).astype(np.int64)
    sh = np.maximum(ebits - 134, -122)
    inv = ((127 - sh).astype(np.uint32) << np.uint32(23)).view(np.float32)
    xs = (x * inv[..., None]).astype(np.float32)
    hi = f32_to_e4m3(xs)
    r = ((xs - e4m3_to_f32(hi)) * np.float32(2.0 ** LO_SHIFT)).astype(np.float32)
    lo = f32_to_e4m3(r)
    return hi.reshape(rows, cols), lo.reshape(rows, cols), (sh + 127).astype(np.uint8)


def join_e4m3(hi, lo, scales):
    """Inverse of ``split_e4m3``: float32 values 2^(s-127) * (hi + 2^-5 * lo)."""
    hi = np.asarray(hi, np.uint8)
    rows, cols = hi.shape
    s = np.asarray(scales, np.int64).repeat(32, axis=1)
    v = e4m3_to_f32(hi).astype(np.float64) + e4m3_to_f32(lo).astype(np.float64) * 2.0 ** -LO_SHIFT
    return (v * np.exp2((s - 127).astype(np.float64))).astype(np.float32)


def kv_scores(query_f32, payload, scales, fmt: int, D: int) -> np.ndarray:
    """MXFP8PoolingCache.quantized_matmul / index_matmul over completed chunks
    (fp8_cache.py:119-159): query [B, Lq, D] @ dequant(K)^T for K [B, L, D]
    stored as MXFP8 / MXFP4 rows, accumulated in float64, rounded to bf16 (the
    query dtype mx.quantized_matmul returns)."""
    q = np.asarray(query_f32, np.float64)
    B, L = payload.shape[0], payload.shape[1]
    k = kv_dequantize(np.asarray(payload).reshape(B * L, -1), np.asarray(scales).reshape(B * L, -1), fmt, D)
    k = k.reshape(B, L, D).astype(np.float64)
    return round_bf16(np.einsum("bqd,bld->bql", q, k).astype(np.float32))

