"""Expert-slot layout and blob placement of an installed model, restated in numpy.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): checks the device
loader, which places every region of every blob with pitched copies.

Follows runtime/deepseek_v4_ssd/expert_layout.py:8-80 (slot layouts) and
expert_cache.py:416-428 (``_SlotPool.store``: each source region is copied to
its offset in the slot layout) and 456-493 (``_batched_array``: the packed
slots viewed as [expert_count, *region.shape] with stride expert_blob_size).
"""
from __future__ import annotations

import numpy as np


def fused_slot_regions(regions, blob_size: int) -> dict:
    """name -> (shape, offset, length) of the DeepSeek fused slot
    (expert_layout.py:8-66): w3.weight, w1.weight (together w13.weight),
    w2.weight, then w3.scale, w1.scale (together w13.scale), w2.scale."""
    src = {r[0]: r for r in regions}
    if set(src) != {"w1.weight", "w1.scale", "w2.weight", "w2.scale", "w3.weight", "w3.scale"}:
        raise ValueError("expert blob does not contain the required regions")
    out, off = {}, 0

    def add(name):
        nonlocal off
        _, _, shape, _, length = src[name]
        out[name] = (tuple(shape), off, length)
        off += length

    add("w3.weight")
    add("w1.weight")
    w3, w1 = src["w3.weight"], src["w1.weight"]
    out["w13.weight"] = ((w3[2][0] + w1[2][0], *w3[2][1:]), 0, w3[4] + w1[4])
    add("w2.weight")
    scale0 = off
    add("w3.scale")
    add("w1.scale")
    s3, s1 = src["w3.scale"], src["w1.scale"]
    out["w13.scale"] = ((s3[2][0] + s1[2][0], *s3[2][1:]), scale0, s3[4] + s1[4])
    add("w2.scale")
    if off != blob_size:
        raise ValueError("fused expert slot size does not match the manifest")
    return out


def qwen_slot_regions(regions, blob_size: int) -> dict:
    """Qwen slots keep the blob layout (expert_layout.py:69-80)."""
    src = {r[0]: r for r in regions}
    if set(src) != {"gate_up.weight", "gate_up.scale", "down.weight", "down.scale"}:
        raise ValueError("Qwen expert blob does not contain the required regions")
    if sum(r[4] for r in regions) != blob_size:
        raise ValueError("Qwen expert slot size does not match the manifest")
    return {r[0]: (tuple(r[2]), r[3], r[4]) for r in regions}


def store(blobs: np.ndarray, regions, slot_regions: dict) -> np.ndarray:
    """Packed slots [E, blob_size] uint8 from the raw blobs [E, blob_size]
    (expert_cache.py:416-428: region by region into the slot layout)."""
    slots = np.zeros_like(blobs)
    for name, _, _, offset, length in regions:
        _, dst, _ = slot_regions[name]
        slots[:, dst:dst + length] = blobs[:, offset:offset + length]
    return slots


def batched(slots: np.ndarray, slot_regions: dict, name: str, dtype: str) -> np.ndarray:
    """[E, *shape] bytes of one slot region (expert_cache.py:456-493); U32
    regions are returned as their little-endian bytes, 4 per word."""
    shape, offset, length = slot_regions[name]
    rows = slots[:, offset:offset + length]
    last = shape[-1] * 4 if dtype == "U32" else shape[-1]
    return rows.reshape(slots.shape[0], *shape[:-1], last)
