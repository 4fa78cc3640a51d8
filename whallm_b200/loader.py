"""Installed-model expert layers -> HBM-resident expert tensors.

An installed model stores each MoE layer as ``experts/layer_XX.bin``:
``expertCount`` blobs of ``expertBlobSize`` bytes, each holding the regions
that ``manifest.json``'s ``expertRegions`` lists (name, dtype, shape, byte
offset, length; runtime/deepseek_v4_ssd/manifest.py:14-47, 150-196).  The
reference's expert cache streams blobs into slots and re-lays them so that a
slot holds ``w13 = [w3; w1]`` and ``w13.scale = [w3.scale; w1.scale]``
(expert_layout.py:8-66, expert_cache.py:416-428); Qwen slots keep
``gate_up``/``down`` as stored (expert_layout.py:69-80).

Here a whole layer becomes resident in one call of ``wld_load_expert_layer``:
the library reads the file through two pinned buffers and places each region
of every blob with one pitched host-to-device copy, straight into the
``[E, ...]`` tensors the expert kernels read.  The result is the
``BatchedExperts`` / ``QwenBatchedExperts`` of ``experts.py``.
"""
from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass
from pathlib import Path

import torch

from . import _lib as L
from . import experts as X

# The pinned blob contracts (manifest.py:21-43): (name, dtype, shape, offset, length).
DEEPSEEK_V4_REGIONS = (
    ("w1.weight", "I8", (2048, 2048), 0, 4194304),
    ("w1.scale", "F8_E8M0", (2048, 128), 4194304, 262144),
    ("w2.weight", "I8", (4096, 1024), 4456448, 4194304),
    ("w2.scale", "F8_E8M0", (4096, 64), 8650752, 262144),
    ("w3.weight", "I8", (2048, 2048), 8912896, 4194304),
    ("w3.scale", "F8_E8M0", (2048, 128), 13107200, 262144),
)
DEEPSEEK_V41_REGIONS = (
    ("w1.weight", "I8", (2304, 2560), 0, 5898240),
    ("w1.scale", "F8_E8M0", (2304, 160), 5898240, 368640),
    ("w2.weight", "I8", (5120, 1152), 6266880, 5898240),
    ("w2.scale", "F8_E8M0", (5120, 72), 12165120, 368640),
    ("w3.weight", "I8", (2304, 2560), 12533760, 5898240),
    ("w3.scale", "F8_E8M0", (2304, 160), 18432000, 368640),
)
QWEN_REGIONS = (
    ("gate_up.weight", "U32", (1280, 320), 0, 1638400),
    ("gate_up.scale", "U8", (1280, 80), 1638400, 102400),
    ("down.weight", "U32", (2560, 80), 1740800, 819200),
    ("down.scale", "U8", (2560, 20), 2560000, 51200),
)
CONTRACTS = {"deepseek-v4": DEEPSEEK_V4_REGIONS, "deepseek-v4.1": DEEPSEEK_V41_REGIONS,
             "qwen3.8-flash-next": QWEN_REGIONS}

_FUSED = {"w1.weight", "w1.scale", "w2.weight", "w2.scale", "w3.weight", "w3.scale"}
_QWEN = {"gate_up.weight", "gate_up.scale", "down.weight", "down.scale"}
_ITEM = {"I8": 1, "U8": 1, "F8_E8M0": 1, "U32": 4}


@dataclass(frozen=True)
class ExpertLayout:
    """What one installed layer file holds."""
    expert_count: int
    blob_size: int
    regions: tuple          # ((name, dtype, shape, offset, length), ...)
    layer_count: int = 0


def read_layout(root) -> ExpertLayout:
    """Expert layout of an installed model's ``manifest.json`` (manifest.py:150-196)."""
    raw = json.loads((Path(root) / "manifest.json").read_text())
    regions = tuple((r["name"], r["dtype"], tuple(r["shape"]), int(r["offset"]), int(r["length"]))
                    for r in raw["expertRegions"])
    return ExpertLayout(int(raw["expertCount"]), int(raw["expertBlobSize"]), regions, int(raw["layerCount"]))


def contract_of(regions) -> str | None:
    """The pinned model contract these regions match, or None."""
    regions = tuple((n, d, tuple(s), o, ln) for n, d, s, o, ln in regions)
    for kind, want in CONTRACTS.items():
        if regions == want:
            return kind
    return None


def _bytes_shape(dtype, shape):
    # every region holds bytes here: a U32 row of w words is 4w bytes
    shape = tuple(shape)
    return (*shape[:-1], shape[-1] * _ITEM[dtype])


def _check_region(name, dtype, shape, offset, length, blob_size):
    if dtype not in _ITEM:
        raise ValueError(f"region {name} has an unsupported dtype {dtype}")
    n = 1
    for v in _bytes_shape(dtype, shape):
        n *= v
    if n != length:
        raise ValueError(f"region {name} length does not match its shape")
    if offset < 0 or offset + length > blob_size:
        raise ValueError(f"region {name} lies outside the blob")


def plan(layout: ExpertLayout, device):
    """Allocate the resident tensors of one layer and the copy plan:
    (tensors, [(src_offset, length, dst_tensor, byte offset within one expert)])."""
    E, blob = layout.expert_count, layout.blob_size
    by = {r[0]: r for r in layout.regions}
    if len(by) != len(layout.regions):
        raise ValueError("expert regions repeat a name")
    for r in layout.regions:
        _check_region(*r, blob)

    def alloc(*rows_then_cols):
        return torch.empty((E, *rows_then_cols), dtype=torch.uint8, device=device)

    if set(by) == _FUSED:
        # the fused slot of expert_layout.py:20-63: w13 = [w3; w1], w13.scale = [w3.scale; w1.scale]
        w1, w3, s1, s3 = by["w1.weight"], by["w3.weight"], by["w1.scale"], by["w3.scale"]
        if w1[1] != w3[1] or w1[2][1:] != w3[2][1:]:
            raise ValueError("w1 and w3 weights cannot use one fused projection")
        if s1[1] != s3[1] or s1[2][1:] != s3[2][1:]:
            raise ValueError("w1 and w3 scales cannot use one fused projection")
        if sum(r[4] for r in layout.regions) != blob:
            raise ValueError("fused expert slot size does not match the manifest")
        w3b, s3b = _bytes_shape(w3[1], w3[2]), _bytes_shape(s3[1], s3[2])
        w13 = alloc(w3b[0] + w1[2][0], *w3b[1:])
        s13 = alloc(s3b[0] + s1[2][0], *s3b[1:])
        w2 = alloc(*_bytes_shape(*by["w2.weight"][1:3]))
        s2 = alloc(*_bytes_shape(*by["w2.scale"][1:3]))
        place = {"w3.weight": (w13, 0), "w1.weight": (w13, w3[4]), "w3.scale": (s13, 0),
                 "w1.scale": (s13, s3[4]), "w2.weight": (w2, 0), "w2.scale": (s2, 0)}
        result = X.BatchedExperts(None, None, w2, s2, None, None, w13, s13)
    elif set(by) == _QWEN:
        if sum(r[4] for r in layout.regions) != blob:
            raise ValueError("Qwen expert slot size does not match the manifest")
        t = {n: alloc(*_bytes_shape(*by[n][1:3])) for n in _QWEN}
        place = {n: (t[n], 0) for n in _QWEN}
        result = X.QwenBatchedExperts(t["gate_up.weight"], t["gate_up.scale"], t["down.weight"], t["down.scale"])
    else:
        raise ValueError("expert blob does not contain a known region set")
    copies = []
    for name, _, _, offset, length in layout.regions:
        dst, at = place[name]
        if at + length > dst[0].numel():
            raise ValueError(f"region {name} does not fit its destination")
        copies.append((offset, length, dst, at))
    return result, copies


def load_expert_layer(path, layout: ExpertLayout, device="cuda", chunk_bytes: int = 256 << 20):
    """Read one installed ``experts/layer_XX.bin`` into resident expert tensors
    on ``device`` (BatchedExperts with w13 = [w3; w1], or QwenBatchedExperts).
    Raises ValueError for a wrong file size or region set (manifest.py:170-175,
    expert_layout.py:18-27)."""
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("experts load onto a CUDA device (no CPU fallback)")
    result, copies = plan(layout, device)
    n = len(copies)
    src = (ctypes.c_size_t * n)(*[c[0] for c in copies])
    lengths = (ctypes.c_size_t * n)(*[c[1] for c in copies])
    bases = (ctypes.c_void_p * n)(*[c[2].data_ptr() + c[3] for c in copies])
    pitches = (ctypes.c_size_t * n)(*[c[2].stride(0) for c in copies])
    with torch.cuda.device(device):
        stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        L.call("wld_load_expert_layer", str(path).encode(), layout.blob_size, layout.expert_count, n, src, lengths,
               bases, pitches, int(chunk_bytes), stream)
    return result


def load_installed_experts(root, layers=None, device="cuda", require_contract: bool = True):
    """The expert layers of an installed model (all, or ``layers``) as a
    ResidentExpertStore.  With ``require_contract`` the manifest's regions must
    be one of the pinned model contracts, as InstalledModel.open requires
    (manifest.py:190-195)."""
    layout = read_layout(root)
    if require_contract and contract_of(layout.regions) is None:
        raise ValueError("installed expert blob layout does not match the model contract")
    store = X.ResidentExpertStore()
    for li in (range(layout.layer_count) if layers is None else layers):
        store.add_layer(li, load_expert_layer(Path(root) / "experts" / f"layer_{li:02d}.bin", layout, device))
    return store
