"""Qwen QSA affine-quantized KV cache on the device.

Mirrors ``QSAQuantizedCache`` (runtime/deepseek_v4_ssd/qwen_quantized_cache.py:6-57),
itself mlx-lm's ``QuantizedKVCache`` with group 32 and 4 or 8 bits: every
``update_and_fetch`` quantizes the new keys and values into the packed
history and returns the whole history dequantized; the retained history stays
packed.  Here both halves are one launch each (``wkv_affine_append``,
``wkv_affine_fetch``, keys and values together).

Storage per tensor: packed uint32 [B, H, capacity, D*bits/32] and bf16 scales
and biases [B, H, capacity, D/32], grown in steps of 256 rows like mlx-lm's
cache, or allocated once at ``capacity`` rows so that the buffers never move.
"""
from __future__ import annotations

import torch

from . import _lib as L

STEP = 256
_SCALE_DTYPES = (torch.bfloat16, torch.float16, torch.float32)   # admitted by the reference


class QSAQuantizedCache:
    def __init__(self, bits: int, dimension: int, capacity: int = 0):
        if bits not in (4, 8) or dimension % 32:
            raise ValueError("QSA quantized cache requires 4 or 8 bits and a width divisible by 32")
        self.bits = bits
        self.group_size = 32
        self.dimension = dimension
        self.offset = 0
        self.keys = None      # (packed, scales, biases), each [B, H, capacity, width]
        self.values = None
        self._reserve = int(capacity)

    # ------------------------------------------------------------ storage --
    def _alloc(self, B, H, rows, device):
        w = self.dimension * self.bits // 32
        g = self.dimension // 32
        return tuple((torch.empty((B, H, rows, w), dtype=torch.int32, device=device),
                      torch.zeros((B, H, rows, g), dtype=torch.bfloat16, device=device),
                      torch.zeros((B, H, rows, g), dtype=torch.bfloat16, device=device)) for _ in range(2))

    def _grow(self, B, H, n, device):
        cap = 0 if self.keys is None else self.keys[0].shape[2]
        if self.keys is not None and self.offset + n <= cap:
            return
        need = self.offset + n
        rows = max(self._reserve, ((need + STEP - 1) // STEP) * STEP)
        k, v = self._alloc(B, H, rows, device)
        if self.keys is not None and self.offset:
            for new, old in zip(k + v, self.keys + self.values):
                new[:, :, :self.offset].copy_(old[:, :, :self.offset])
        self.keys, self.values = k, v

    # ------------------------------------------------------------- update --
    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor):
        """keys, values bf16 [B, H, L, D] -> the dequantized history (keys, values) bf16 [B, H, offset, D]."""
        if keys.shape[-1] != self.dimension or values.shape[-1] != self.dimension:
            raise ValueError("QSA cache width does not match")
        if keys.dtype != torch.bfloat16 or values.dtype != torch.bfloat16:
            raise ValueError("QSA cache takes bf16 keys and values")
        if keys.shape != values.shape or keys.dim() != 4:
            raise ValueError("QSA cache keys and values must be [B, H, L, D] of one shape")
        B, H, n, D = keys.shape
        if self.keys is not None and tuple(self.keys[0].shape[:2]) != (B, H):
            raise ValueError("QSA cache batch or head count changed")
        k = keys.contiguous()
        v = values.contiguous()
        L.require_cuda(k, v)
        self._grow(B, H, n, k.device)
        cap = self.keys[0].shape[2]
        st = L.stream_of(k)
        (kq, ks, kb), (vq, vs, vb) = self.keys, self.values
        L.call("wkv_affine_append", L.ptr(k), L.ptr(v), B * H, n, D, self.bits, L.ptr(kq), L.ptr(ks), L.ptr(kb),
               L.ptr(vq), L.ptr(vs), L.ptr(vb), cap, self.offset, st)
        self.offset += n
        return self.fetch()

    def fetch(self):
        """The dequantized history (keys, values) bf16 [B, H, offset, D]."""
        (kq, ks, kb), (vq, vs, vb) = self.keys, self.values
        B, H, cap, _ = kq.shape
        ko = torch.empty((B, H, self.offset, self.dimension), dtype=torch.bfloat16, device=kq.device)
        vo = torch.empty_like(ko)
        L.call("wkv_affine_fetch", L.ptr(kq), L.ptr(ks), L.ptr(kb), L.ptr(vq), L.ptr(vs), L.ptr(vb), B * H,
               self.offset, cap, self.dimension, self.bits, L.ptr(ko), L.ptr(vo), L.stream_of(kq))
        return ko, vo

    # -------------------------------------------------------- persistence --
    @property
    def state(self):
        """The packed history, trimmed to ``offset`` rows (mlx-lm QuantizedKVCache.state)."""
        return tuple(tuple(a[:, :, :self.offset] for a in part) for part in (self.keys, self.values))

    def persistence_state(self):
        return dict(bits=self.bits, dimension=self.dimension, offset=self.offset,
                    arrays=self.state if self.keys is not None else None)

    def restore_persistence_state(self, saved):
        """Adopt a saved state after the checks of qwen_quantized_cache.py:26-57."""
        if (not isinstance(saved, dict) or set(saved) != {"bits", "dimension", "offset", "arrays"}
                or saved["bits"] != self.bits or saved["dimension"] != self.dimension
                or type(saved["offset"]) is not int or saved["offset"] < 0):
            raise ValueError("Invalid QSA packed cache format")
        arrays, offset = saved["arrays"], saved["offset"]
        if arrays is None:
            if offset:
                raise ValueError("Empty QSA cache has nonzero offset")
            self.keys = self.values = None
            self.offset = 0
            return
        if not isinstance(arrays, (list, tuple)) or len(arrays) != 2:
            raise ValueError("Invalid QSA packed cache arrays")
        first = None
        for item in arrays:
            if not isinstance(item, (tuple, list)) or len(item) != 3:
                raise ValueError("Invalid QSA packed cache component")
            for i, a in enumerate(item):
                width = self.dimension * self.bits // 32 if i == 0 else self.dimension // 32
                if (not isinstance(a, torch.Tensor) or a.dim() != 4 or a.shape[0] != 1
                        or tuple(a.shape[2:]) != (offset, width)
                        or (i == 0 and a.dtype not in (torch.int32, torch.uint32))
                        or (i > 0 and a.dtype not in _SCALE_DTYPES)):
                    raise ValueError("Invalid QSA packed cache shape or dtype")
                if first is None:
                    first = tuple(a.shape[:3])
                if tuple(a.shape[:3]) != first:
                    raise ValueError("QSA packed cache components do not match")
                if i > 0 and a.dtype != torch.bfloat16:
                    # the reference also admits f16/f32 scales; this path stores what a bf16 model writes
                    raise ValueError("QSA packed cache scales and biases must be bf16 here")
        # a private copy, packed words as int32
        self.keys, self.values = [tuple((a.view(torch.int32) if i == 0 else a).contiguous().clone()
                                        for i, a in enumerate(item)) for item in arrays]
        self.offset = offset


# --------------------------------------------------------------------------
# V4.1 packed rows (deepseek_v41/packed_cache.py:8-78)
# --------------------------------------------------------------------------

from . import formats as _F  # noqa: E402

_PACKED_KINDS = {"fp8_ue8m0": (32, 8), "fp4_e4m3": (16, 4), "fp4_ue8m0": (32, 4)}


class PackedRows:
    """V4.1 activation rows stored as bytes on the device: e4m3 or e2m1 payload
    plus one scale byte per block, written once with the checkpoint's scale
    rules (``wkv_quantize``) and read back with ``wkv_dequantize``; indexes
    address the leading dimensions as in the reference (slices, integer and
    index-tensor selections)."""

    def __init__(self, shape, kind, dtype=torch.bfloat16, device="cuda"):
        self.shape = tuple(shape)
        self.kind = kind
        self.dtype = dtype
        if kind not in _PACKED_KINDS or self.shape[-1] % _PACKED_KINDS[kind][0]:
            raise ValueError("Invalid V4.1 packed cache format or width")
        self.block, self.bits = _PACKED_KINDS[kind]
        self.payload = torch.zeros((*self.shape[:-1], self.shape[-1] * self.bits // 8), dtype=torch.uint8,
                                   device=device)
        self.scales = torch.zeros((*self.shape[:-1], self.shape[-1] // self.block), dtype=torch.uint8, device=device)

    @property
    def nbytes(self):
        return self.payload.numel() + self.scales.numel()

    def write(self, index, value):
        """Quantize ``value`` (the rows at ``index``) once and store the bytes."""
        v = value.to(torch.bfloat16).contiguous()
        p, s = _F.kv_quantize(v, self.kind)
        self.payload[index] = p
        self.scales[index] = s

    def __getitem__(self, index):
        p = self.payload[index].contiguous()
        s = self.scales[index].contiguous()
        out = _F.kv_dequantize(p, s, self.kind)
        return out if self.dtype == torch.bfloat16 else out.to(self.dtype)

    def grow(self, capacity):
        enlarged = PackedRows((self.shape[0], capacity, self.shape[2]), self.kind, self.dtype, self.payload.device)
        enlarged.payload[:, :self.shape[1]] = self.payload
        enlarged.scales[:, :self.shape[1]] = self.scales
        return enlarged

    def state(self):
        return dict(format=self.kind, payload=self.payload, scales=self.scales)

    def restore(self, state):
        if not isinstance(state, dict) or set(state) != {"format", "payload", "scales"} or state["format"] != self.kind:
            raise ValueError("V4.1 packed cache format does not match")
        for name in ("payload", "scales"):
            saved, expected = state[name], getattr(self, name)
            if (not isinstance(saved, torch.Tensor) or tuple(saved.shape) != tuple(expected.shape)
                    or saved.dtype != torch.uint8):
                raise ValueError("Invalid V4.1 packed cache array")
        self.payload = state["payload"].to(self.payload.device).clone()
        self.scales = state["scales"].to(self.scales.device).clone()
        return self


# --------------------------------------------------------------------------
# MXFP8 pooled (compressed-attention) cache (fp8_cache.py:59-240)
# --------------------------------------------------------------------------

class MXFP8PoolingCache:
    """Completed 64-row chunks of the compressed-attention cache stored as
    MXFP8 (e4m3 + E8M0 per 32) and, for the indexer, an MXFP4 copy; the rows
    of an incomplete chunk stay bf16 (``pending``), as in fp8_cache.py:94-117.
    Storage is one device buffer per format, [B, capacity, ...], grown by
    doubling; scores over the completed rows run on the block-scaled tensor
    cores (``wkv_mx_scores``), gathers through ``wkv_gather_dequantize``.

    The mlx-lm PoolingCache window machinery (``accumulate_windows`` and the
    raw window buffers) belongs to the attention compressor, not to this
    cache's quantized storage, and is not reproduced: ``state`` carries
    ``None`` in those positions."""

    chunk_size = 64
    fp4_index = True

    def __init__(self, ratio: int, device="cuda"):
        self.ratio = ratio
        self.device = torch.device(device)
        self._pending = None
        self._length = 0
        self._completed = 0                 # rows in the quantized buffers
        self._last_shape = None
        self._q8 = self._s8 = self._q4 = self._s4 = None
        self.previous_window_kv = self.previous_window_gate = None

    # ------------------------------------------------------------ storage --
    @property
    def offset(self):
        return self._length

    @property
    def shape(self):
        batch, width = self._last_shape or (1, 0)
        return batch, self._length, width

    @property
    def nbytes(self):
        n = sum(t.numel() for t in (self._q8, self._s8, self._q4, self._s4) if t is not None)
        return n + (self._pending.numel() * self._pending.element_size() if self._pending is not None else 0)

    def _reserve(self, B, D, rows):
        cap = 0 if self._q8 is None else self._q8.shape[1]
        if rows <= cap:
            return
        new = max(rows, 2 * cap, 4 * self.chunk_size)
        dev = self.device
        q8 = torch.empty((B, new, D), dtype=torch.uint8, device=dev)
        s8 = torch.empty((B, new, D // 32), dtype=torch.uint8, device=dev)
        q4 = torch.empty((B, new, D // 2), dtype=torch.uint8, device=dev) if self.fp4_index else None
        s4 = torch.empty((B, new, D // 32), dtype=torch.uint8, device=dev) if self.fp4_index else None
        n = self._completed
        if n:
            q8[:, :n] = self._q8[:, :n]
            s8[:, :n] = self._s8[:, :n]
            if q4 is not None:
                q4[:, :n] = self._q4[:, :n]
                s4[:, :n] = self._s4[:, :n]
        self._q8, self._s8, self._q4, self._s4 = q8, s8, q4, s4

    def update(self, px):
        """Append rows px [B, L, D]; every completed 64-row chunk is quantized
        (mxfp8, and mxfp4 for the index copy) into the buffers."""
        if px.shape[1] == 0:
            return
        B, L, D = px.shape
        if D % 32:
            raise ValueError("MXFP8 pooling cache width must be a multiple of 32")
        self._last_shape = (B, D)
        self._length += L
        self._pending = px if self._pending is None else torch.cat([self._pending, px], dim=1)
        ready = self._pending.shape[1] // self.chunk_size * self.chunk_size
        if not ready:
            return
        done = self._pending[:, :ready].to(torch.bfloat16).contiguous()
        self._pending = self._pending[:, ready:] if ready < self._pending.shape[1] else None
        n = self._completed
        self._reserve(B, D, n + ready)
        for b in range(B):      # rows of one sequence are contiguous in the buffers
            _F.kv_quantize(done[b], "mxfp8", self._q8[b, n:n + ready], self._s8[b, n:n + ready])
            if self.fp4_index:
                _F.kv_quantize(done[b], "mxfp4", self._q4[b, n:n + ready], self._s4[b, n:n + ready])
        self._completed = n + ready

    def update_and_fetch(self, px):
        self.update(px)
        return self.fetch(px.shape[0], px.shape[-1], px.dtype)

    # ------------------------------------------------------------- scores --
    def _scores(self, query, q, s, fmt):
        B, D = self._last_shape
        n = self._completed
        lead = query.shape[:-1]
        q3 = query.reshape(B, -1, D)
        if D % 256 == 0:
            out = torch.empty((B, q3.shape[1], n), dtype=torch.bfloat16, device=query.device)
            for b in range(B):
                _F.kv_scores(q3[b:b + 1].to(torch.bfloat16).contiguous(), q[b:b + 1, :n].contiguous(),
                             s[b:b + 1, :n].contiguous(), fmt, out=out[b:b + 1])
            return out.to(query.dtype).reshape(*lead, n)
        # widths the tensor-core score kernel does not tile (D % 256 != 0): the
        # rows are dequantized on the device, then one library GEMM in f32
        rows = torch.stack([_F.kv_dequantize(q[b, :n].contiguous(), s[b, :n].contiguous(), fmt) for b in range(B)])
        return (q3.float() @ rows.float().transpose(-1, -2)).to(query.dtype).reshape(*lead, n)

    def _pending_scores(self, query):
        B, D = self._last_shape
        q3 = query.reshape(B, -1, D)
        sc = q3 @ self._pending.to(query.dtype).transpose(-1, -2)
        return sc.reshape(*query.shape[:-1], self._pending.shape[1])

    def quantized_matmul(self, query):
        """query [B, ..., D] against every cached row -> [B, ..., rows]."""
        parts = []
        if self._completed:
            parts.append(self._scores(query, self._q8, self._s8, "mxfp8"))
        if self._pending is not None:
            parts.append(self._pending_scores(query))
        if not parts:
            return torch.zeros((*query.shape[:-1], 0), dtype=query.dtype, device=query.device)
        return parts[0] if len(parts) == 1 else torch.cat(parts, dim=-1)

    def index_matmul(self, query):
        if not self.fp4_index or not self._completed:
            return self.quantized_matmul(query)
        parts = [self._scores(query, self._q4, self._s4, "mxfp4")]
        if self._pending is not None:
            parts.append(self._pending_scores(query))
        return parts[0] if len(parts) == 1 else torch.cat(parts, dim=-1)

    # ------------------------------------------------------------- gather --
    def gather(self, indices):
        """indices [B, L, k] -> rows [B, L, k, D] (fp8_cache.py:161-202)."""
        B, D = self._last_shape
        n = self._completed
        completed = None
        if n:
            cap = self._q8.shape[1]
            rows = indices.to(torch.int64).clamp(0, n - 1)
            flat = (rows + torch.arange(B, device=indices.device).view(B, 1, 1) * cap).to(torch.int32).contiguous()
            completed = _F.kv_gather_dequantize(self._q8.view(B * cap, D), self._s8.view(B * cap, D // 32), flat,
                                                "mxfp8")
        if self._pending is None:
            return completed
        P = self._pending.shape[1]
        prow = (indices.to(torch.int64) - n).clamp(0, P - 1)
        pending = torch.gather(self._pending.unsqueeze(1).expand(B, indices.shape[1], P, D), 2,
                               prow.unsqueeze(-1).expand(*prow.shape, D))
        if completed is None:
            return pending
        return torch.where((indices >= n).unsqueeze(-1), pending, completed.to(pending.dtype))

    # -------------------------------------------------------------- fetch --
    def fetch(self, batch, width, dtype):
        parts = []
        if self._completed:
            n = self._completed
            parts.append(torch.stack([_F.kv_dequantize(self._q8[b, :n].contiguous(), self._s8[b, :n].contiguous(),
                                                       "mxfp8") for b in range(self._q8.shape[0])]).to(dtype))
        if self._pending is not None:
            parts.append(self._pending.to(dtype))
        if parts:
            return parts[0] if len(parts) == 1 else torch.cat(parts, dim=1)
        return torch.zeros((batch, 0, width), dtype=dtype, device=self.device)

    def __getitem__(self, key):
        batch, width = self._last_shape
        dtype = self._pending.dtype if self._pending is not None else torch.bfloat16
        return self.fetch(batch, width, dtype)[key]

    def make_mask(self, length: int = 1, offset: int = 0):
        if self._length == 0 or length == 1:
            return None
        pool_index = torch.arange(self._length, device=self.device)
        query_index = torch.arange(offset + 1, offset + length + 1, device=self.device)
        return pool_index < (query_index[:, None] // self.ratio)

    # -------------------------------------------------------------- state --
    @property
    def state(self):
        pooled = None
        if self._length:
            batch, width = self._last_shape
            dtype = self._pending.dtype if self._pending is not None else torch.bfloat16
            pooled = self.fetch(batch, width, dtype)
        return None, None, pooled, self.previous_window_kv, self.previous_window_gate

    @state.setter
    def state(self, value):
        if len(value) == 3:
            buf_kv, buf_gate, pooled = value
            previous_kv = previous_gate = None
        elif len(value) == 5:
            buf_kv, buf_gate, pooled, previous_kv, previous_gate = value
        else:
            raise ValueError("MXFP8 pooling cache state must have 3 or 5 values")
        if buf_kv is not None or buf_gate is not None:
            raise ValueError("MXFP8 pooling cache: raw window buffers are kept by the attention compressor")
        self._pending = None
        self._length = self._completed = 0
        self._last_shape = None
        self._q8 = self._s8 = self._q4 = self._s4 = None
        self.previous_window_kv, self.previous_window_gate = previous_kv, previous_gate
        if pooled is not None:
            self.update_and_fetch(pooled)
