"""Installed-model expert loader: manifest regions -> resident expert tensors.

CPU: the copy plan reproduces the reference's slot layout and store
(oracle/loader.py, after expert_layout.py:8-80 and expert_cache.py:416-493)
byte for byte, bad region sets are rejected as the reference rejects them,
and the native loader refuses a file of the wrong size before any CUDA call.

GPU: synthetic installed models in the pinned DeepSeek V4, V4.1 and Qwen blob
contracts are written in the reference's file layout, loaded through
``wld_load_expert_layer`` (with chunk sizes that give one blob per chunk and a
ragged last chunk), and the resident tensors equal the oracle's batched slots
bit for bit; an MoE forward on the loaded experts equals the forward on the
experts the file was written from, bit for bit.
"""
import ctypes
import json

import numpy as np
import pytest
import torch

import whallm_b200 as W
from oracle import loader as OL
from whallm_b200 import _lib as L
from whallm_b200 import loader as LD
from whallm_b200 import synthetic as S

# a small fused layout: H = 64, I = 32 (w1/w3 [I, H/2], w2 [H, I/2], scales per 32)
SMALL = (
    ("w1.weight", "I8", (32, 32), 0, 1024),
    ("w1.scale", "F8_E8M0", (32, 2), 1024, 64),
    ("w2.weight", "I8", (64, 16), 1088, 1024),
    ("w2.scale", "F8_E8M0", (64, 1), 2112, 64),
    ("w3.weight", "I8", (32, 32), 2176, 1024),
    ("w3.scale", "F8_E8M0", (32, 2), 3200, 64),
)


def _emulate(copies, blobs):
    """Apply the copy plan on the CPU (what the pitched copies do on the device)."""
    E = blobs.shape[0]
    for src, length, dst, at in copies:
        rows = dst.view(E, -1)
        rows[:, at:at + length] = torch.from_numpy(blobs[:, src:src + length].copy())


def _oracle_tensors(regions, blobs, qwen):
    blob = blobs.shape[1]
    dt = {r[0]: r[1] for r in regions}
    if qwen:
        sr = OL.qwen_slot_regions(regions, blob)
        names = ("gate_up.weight", "gate_up.scale", "down.weight", "down.scale")
    else:
        sr = OL.fused_slot_regions(regions, blob)
        dt["w13.weight"], dt["w13.scale"] = dt["w3.weight"], dt["w3.scale"]
        names = ("w13.weight", "w13.scale", "w2.weight", "w2.scale")
    slots = OL.store(blobs, regions, sr)
    return [OL.batched(slots, sr, n, dt[n]) for n in names]


def _loaded_tensors(b):
    if isinstance(b, W.QwenBatchedExperts):
        return [b.gate_up, b.gate_up_scales, b.down, b.down_scales]
    return [b.w13, b.w13_scales, b.w2, b.w2_scales]


def test_fused_slot_layout_of_the_deepseek_contract():
    sr = OL.fused_slot_regions(LD.DEEPSEEK_V4_REGIONS, 13_369_344)
    assert sr["w3.weight"][1:] == (0, 4_194_304)
    assert sr["w1.weight"][1:] == (4_194_304, 4_194_304)
    assert sr["w13.weight"] == ((4096, 2048), 0, 8_388_608)
    assert sr["w2.weight"][1] == 8_388_608
    assert sr["w13.scale"] == ((4096, 128), 12_582_912, 524_288)
    assert sr["w2.scale"][1] == 13_107_200
    assert LD.contract_of(LD.DEEPSEEK_V4_REGIONS) == "deepseek-v4"
    assert LD.contract_of(LD.QWEN_REGIONS) == "qwen3.8-flash-next"
    assert LD.contract_of(SMALL) is None


@pytest.mark.parametrize("regions,qwen", [(SMALL, False), (LD.QWEN_REGIONS, True)])
def test_copy_plan_matches_slot_store(regions, qwen):
    blob = sum(r[4] for r in regions)
    E = 3
    blobs = np.random.default_rng(5).integers(0, 256, (E, blob), dtype=np.uint8)
    result, copies = LD.plan(LD.ExpertLayout(E, blob, regions), "cpu")
    _emulate(copies, blobs)
    for got, want in zip(_loaded_tensors(result), _oracle_tensors(regions, blobs, qwen)):
        assert tuple(got.shape) == want.shape
        np.testing.assert_array_equal(got.numpy(), want)


def test_plan_shapes_of_the_deepseek_contract():
    result, copies = LD.plan(LD.ExpertLayout(1, 13_369_344, LD.DEEPSEEK_V4_REGIONS), "cpu")
    assert tuple(result.w13.shape) == (1, 4096, 2048)
    assert tuple(result.w13_scales.shape) == (1, 4096, 128)
    assert tuple(result.w2.shape) == (1, 4096, 1024)
    assert tuple(result.w2_scales.shape) == (1, 4096, 64)
    assert len(copies) == 6


@pytest.mark.parametrize("mutate,msg", [
    (lambda r: r[:-1], "known region set"),
    (lambda r: r[:4] + (("w3.weight", "I8", (32, 16), 2176, 512), r[5]), "fused projection"),
    (lambda r: r[:1] + (("w1.scale", "F8_E8M0", (32, 2), 1024, 60),) + r[2:], "length does not match"),
    (lambda r: r[:5] + (("w3.scale", "F8_E8M0", (32, 2), 3230, 64),), "outside the blob"),
])
def test_plan_rejects_bad_regions(mutate, msg):
    with pytest.raises(ValueError, match=msg):
        LD.plan(LD.ExpertLayout(2, 3264, mutate(SMALL)), "cpu")


def _write_model(root, regions, layers_blobs):
    """An installed model's expert part in the reference's file layout."""
    (root / "experts").mkdir(parents=True, exist_ok=True)
    blob = layers_blobs[0].shape[1]
    for li, b in enumerate(layers_blobs):
        b.tofile(root / "experts" / f"layer_{li:02d}.bin")
    manifest = {"layerCount": len(layers_blobs), "expertCount": layers_blobs[0].shape[0], "expertBlobSize": blob,
                "expertRegions": [{"name": n, "dtype": d, "shape": list(s), "offset": o, "length": ln}
                                  for n, d, s, o, ln in regions]}
    (root / "manifest.json").write_text(json.dumps(manifest))


def test_layout_from_manifest_and_contract_check(tmp_path):
    blobs = np.zeros((2, 3264), np.uint8)
    _write_model(tmp_path, SMALL, [blobs])
    lay = LD.read_layout(tmp_path)
    assert (lay.expert_count, lay.blob_size, lay.layer_count) == (2, 3264, 1)
    assert lay.regions == SMALL
    with pytest.raises(ValueError, match="model contract"):
        LD.load_installed_experts(tmp_path)


def test_native_loader_rejects_wrong_file_size(tmp_path):
    # validated before any CUDA call: runs without a GPU
    p = tmp_path / "layer_00.bin"
    np.zeros(1000, np.uint8).tofile(p)
    n = 1
    src = (ctypes.c_size_t * n)(0)
    ln = (ctypes.c_size_t * n)(100)
    dst = (ctypes.c_void_p * n)(256)      # never dereferenced: the size check fails first
    pitch = (ctypes.c_size_t * n)(100)
    with pytest.raises(ValueError, match="invalid size"):
        L.call("wld_load_expert_layer", str(p).encode(), 300, 3, n, src, ln, dst, pitch, 1 << 20, None)
    with pytest.raises(ValueError, match="cannot open"):
        L.call("wld_load_expert_layer", str(tmp_path / "none.bin").encode(), 100, 10, n, src, ln, dst, pitch,
               1 << 20, None)
    ln[0] = 400
    with pytest.raises(ValueError, match="outside the blob"):
        L.call("wld_load_expert_layer", str(p).encode(), 100, 10, n, src, ln, dst, pitch, 1 << 20, None)


# --------------------------------------------------------------------------
# GPU: load through the C ABI
# --------------------------------------------------------------------------

def _blobs_from_experts(ex, regions, qwen):
    """Serialise resident experts into blobs of the given contract (the inverse of the load)."""
    if qwen:
        parts = {"gate_up.weight": ex.gate_up, "gate_up.scale": ex.gate_up_scales, "down.weight": ex.down,
                 "down.scale": ex.down_scales}
    else:
        I = ex.w13.shape[1] // 2      # w13 = [w3; w1]
        parts = {"w3.weight": ex.w13[:, :I], "w1.weight": ex.w13[:, I:], "w3.scale": ex.w13_scales[:, :I],
                 "w1.scale": ex.w13_scales[:, I:], "w2.weight": ex.w2, "w2.scale": ex.w2_scales}
    E = ex.w2.shape[0] if not qwen else ex.down.shape[0]
    blob = sum(r[4] for r in regions)
    out = np.zeros((E, blob), np.uint8)
    for name, _, _, off, ln in regions:
        out[:, off:off + ln] = parts[name].reshape(E, -1).cpu().numpy()
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("chunk_blobs", [1, 4])
def test_gpu_load_deepseek_layers(dev, tmp_path, chunk_blobs):
    regions, E, H, I = LD.DEEPSEEK_V4_REGIONS, 6, 4096, 2048
    blob = 13_369_344
    src = [S.make_mxfp4_experts(E, H, I, seed=40 + li, device=dev) for li in range(2)]
    blobs = [_blobs_from_experts(ex, regions, False) for ex in src]
    _write_model(tmp_path, regions, blobs)
    lay = LD.read_layout(tmp_path)
    store = LD.load_installed_experts(tmp_path, device=dev)
    for li in range(2):
        got = store.current_batched(li)
        for g, want in zip(_loaded_tensors(got), _oracle_tensors(regions, blobs[li], False)):
            np.testing.assert_array_equal(g.cpu().numpy(), want)
    # chunking: one blob per chunk, or 4 + a ragged 2
    one = LD.load_expert_layer(tmp_path / "experts" / "layer_01.bin", lay, dev, chunk_bytes=chunk_blobs * blob)
    for g, want in zip(_loaded_tensors(one), _loaded_tensors(src[1])):
        assert torch.equal(g, want)
    x = S.make_tokens(5, H, seed=3, device=dev)
    idx = torch.randint(0, E, (5, 4), device=dev, dtype=torch.int32)
    w = torch.rand(5, 4, device=dev)
    a = W.experts_forward(x, idx, one, weights=w, swiglu_limit=10.0)
    b = W.experts_forward(x, idx, src[1], weights=w, swiglu_limit=10.0)
    assert torch.equal(a, b)


@pytest.mark.gpu
def test_gpu_load_qwen_layer(dev, tmp_path):
    regions, E, H, I = LD.QWEN_REGIONS, 8, 2560, 640
    src = S.make_mxfp4_experts(E, H, I, seed=7, device=dev, qwen=True)
    blobs = _blobs_from_experts(src, regions, True)
    _write_model(tmp_path, regions, [blobs])
    got = LD.load_installed_experts(tmp_path, device=dev).current_batched(0)
    assert isinstance(got, W.QwenBatchedExperts)
    for g, want in zip(_loaded_tensors(got), _oracle_tensors(regions, blobs, True)):
        np.testing.assert_array_equal(g.cpu().numpy(), want)
    x = S.make_tokens(3, H, seed=4, device=dev)
    idx = torch.randint(0, E, (3, 2), device=dev, dtype=torch.int32)
    w = torch.rand(3, 2, device=dev)
    assert torch.equal(W.experts_forward(x, idx, got, weights=w), W.experts_forward(x, idx, src, weights=w))


@pytest.mark.gpu
def test_gpu_load_v41_layer_bytes(dev, tmp_path):
    regions = LD.DEEPSEEK_V41_REGIONS
    blob = sum(r[4] for r in regions)
    blobs = np.random.default_rng(11).integers(0, 256, (3, blob), dtype=np.uint8)
    _write_model(tmp_path, regions, [blobs])
    got = LD.load_installed_experts(tmp_path, device=dev).current_batched(0)
    assert tuple(got.w13.shape) == (3, 4608, 2560)
    for g, want in zip(_loaded_tensors(got), _oracle_tensors(regions, blobs, False)):
        np.testing.assert_array_equal(g.cpu().numpy(), want)
