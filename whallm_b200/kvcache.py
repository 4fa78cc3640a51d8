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
