"""HBM-resident routed experts and the grouped expert forward.

Replaces the reference's SSD expert store and its MLX expert math:
  * weight containers with the reference's field names and shapes
    (``ExpertWeights`` / ``BatchedExperts`` / ``QwenExpertWeights`` /
    ``QwenBatchedExperts``, expert_cache.py:31-75), plus the affine-4
    container of the tiny config;
  * ``ResidentExpertStore`` -- the provisioning interface the MoE layer uses
    (``current_batched`` expert_cache.py:990, ``get_many`` :1126,
    ``iter_ready`` :1199, ``prefetch_layer`` :1003, ``batched_layer`` :1058,
    ``record_gather_qmm`` :828), backed by tensors that stay in HBM;
  * ``StreamingSwitchGLU`` -- ``_StreamingSwitchGLU`` (model.py:276-459):
    ``switch_mlp(x, indices) -> [..., k, H]``;
  * ``StreamingExperts`` -- Qwen ``StreamingExperts`` (qwen4_exp.py:600-678);
  * ``experts_forward`` / ``moe_forward`` -- one native call each.

Packed weights are uint8 (MXFP4: two e2m1 per byte, low nibble first;
byte-identical to MLX's uint32 view) or int32 words (affine-4).
"""
from __future__ import annotations

import threading
from contextlib import contextmanager
from dataclasses import dataclass, field

import torch

from . import _lib as L

UP_GATE = L.WM_UP_GATE   # DeepSeek w13 = [w3(up); w1(gate)]
GATE_UP = L.WM_GATE_UP   # Qwen gate_up = [gate; up]


@dataclass(frozen=True)
class ExpertWeights:
    """One DeepSeek expert (expert_cache.py:31-40)."""
    w1: torch.Tensor
    w1_scales: torch.Tensor
    w2: torch.Tensor
    w2_scales: torch.Tensor
    w3: torch.Tensor
    w3_scales: torch.Tensor
    w13: torch.Tensor | None = None
    w13_scales: torch.Tensor | None = None


@dataclass(frozen=True)
class ResidentExperts:
    individual_weights: tuple
    slots: dict


@dataclass(frozen=True)
class BatchedExperts:
    """Stacked DeepSeek experts [E, ...] (expert_cache.py:49-58).  The kernel
    reads w13 ([w3; w1] fused, rows = 2I) and w2."""
    w1: torch.Tensor | None
    w1_scales: torch.Tensor | None
    w2: torch.Tensor
    w2_scales: torch.Tensor
    w3: torch.Tensor | None
    w3_scales: torch.Tensor | None
    w13: torch.Tensor | None = None
    w13_scales: torch.Tensor | None = None

    def fused(self):
        """(w13, w13_scales, gather_qmm calls).  When the store supplied w1 and
        w3 unfused, the [w3; w1] fusion of _fused_slot_regions
        (expert_layout.py:43-62) is built once and kept with this object, not
        rebuilt on every call (a DeepSeek-class layer is ~4 GB of w13)."""
        if self.w13 is not None and self.w13_scales is not None:
            return self.w13, self.w13_scales, 2
        cached = self.__dict__.get("_fused13")
        if cached is None:
            w13 = torch.cat([self.w3, self.w1], dim=-2).contiguous()
            s13 = torch.cat([self.w3_scales, self.w1_scales], dim=-2).contiguous()
            cached = (w13, s13)
            object.__setattr__(self, "_fused13", cached)     # frozen dataclass: a private cache slot
        return cached[0], cached[1], 3


@dataclass(frozen=True)
class QwenExpertWeights:
    gate_up: torch.Tensor
    gate_up_scales: torch.Tensor
    down: torch.Tensor
    down_scales: torch.Tensor


@dataclass(frozen=True)
class QwenBatchedExperts:
    """Stacked Qwen experts (expert_cache.py:69-75): gate_up = [gate; up]."""
    gate_up: torch.Tensor
    gate_up_scales: torch.Tensor
    down: torch.Tensor
    down_scales: torch.Tensor


@dataclass(frozen=True)
class Affine4BatchedExperts:
    """Stacked MLX-affine-4 experts (tiny config): w13 int32 [E, 2I, H/8] with
    bf16 scales/biases [E, 2I, H/group]; w2 int32 [E, H, I/8] + [E, H, I/group]."""
    w13: torch.Tensor
    w13_scales: torch.Tensor
    w13_biases: torch.Tensor
    w2: torch.Tensor
    w2_scales: torch.Tensor
    w2_biases: torch.Tensor
    group: int = 64
    order: int = GATE_UP


@dataclass
class StoreMetrics:
    gather_qmm_calls: int = 0
    expert_calls: int = 0


class ResidentExpertStore:
    """HBM-resident replacement for ExpertCache's provisioning interface.

    ``layers`` maps a layer index to its batched experts (all experts of the
    layer stay resident; there is no eviction)."""

    def __init__(self, layers: dict | None = None):
        self._layers = dict(layers or {})
        self._lock = threading.Lock()
        self.metrics = StoreMetrics()

    def add_layer(self, layer: int, batched) -> None:
        self._layers[layer] = batched

    def current_batched(self, layer: int):
        return self._layers.get(layer)

    def record_gather_qmm(self, calls: int = 3) -> None:
        with self._lock:
            self.metrics.gather_qmm_calls += calls

    def prefetch_layer(self, layer: int, experts=None) -> None:
        """Nothing to read: every expert is resident (expert_cache.py:1003-1017
        checks the same arguments before starting its reads)."""
        if layer not in self._layers:
            return
        if experts is not None and not tuple(experts):
            raise ValueError("batched expert prefetch cannot be empty")

    @contextmanager
    def batched_layer(self, layer: int, enabled: bool = True, experts=None):
        """The layer's batched experts for the duration of the block, or None
        when disabled (expert_cache.py:1058-1067)."""
        if not enabled:
            yield None
            return
        self.prefetch_layer(layer, experts)
        yield self.current_batched(layer)

    def iter_ready(self, layer: int, expert_ids: list):
        """(expert, weights) for each distinct expert, in id order; all are
        ready at once (expert_cache.py:1199-1213)."""
        batched = self._layers.get(layer)
        if batched is None:
            raise ValueError(f"invalid layer {layer}")
        unique = sorted(set(int(e) for e in expert_ids))
        n = _expert_count(batched)
        if any(not 0 <= e < n for e in unique):
            raise ValueError("selected experts contain an invalid expert ID")
        for e in unique:
            yield e, _individual(batched, e)

    def get_many(self, layer: int, expert_ids: list) -> ResidentExperts:
        batched = self._layers.get(layer)
        if batched is None:
            raise ValueError(f"invalid layer {layer}")
        unique = sorted(set(int(e) for e in expert_ids))
        n = _expert_count(batched)
        for e in unique:
            if not 0 <= e < n:
                raise ValueError(f"invalid expert {e}")
        weights = tuple(_individual(batched, e) for e in unique)
        return ResidentExperts(weights, {e: i for i, e in enumerate(unique)})


def _expert_count(b) -> int:
    if isinstance(b, QwenBatchedExperts):
        return b.gate_up.shape[0]
    if isinstance(b, Affine4BatchedExperts):
        return b.w13.shape[0]
    return b.w2.shape[0]


def _individual(b, e):
    if isinstance(b, QwenBatchedExperts):
        return QwenExpertWeights(b.gate_up[e], b.gate_up_scales[e], b.down[e], b.down_scales[e])
    if isinstance(b, Affine4BatchedExperts):
        return Affine4BatchedExperts(b.w13[e:e + 1], b.w13_scales[e:e + 1], b.w13_biases[e:e + 1], b.w2[e:e + 1],
                                     b.w2_scales[e:e + 1], b.w2_biases[e:e + 1], b.group, b.order)
    w13, s13, _ = b.fused()
    pick = lambda t: None if t is None else t[e]
    return ExpertWeights(pick(b.w1), pick(b.w1_scales), b.w2[e], b.w2_scales[e], pick(b.w3), pick(b.w3_scales),
                         w13[e], s13[e])


# --------------------------------------------------------------------------
# workspace
# --------------------------------------------------------------------------

class Workspace:
    """Grow-only device workspace per (device, stream); reused across calls so
    that CUDA-graph captures see stable addresses."""

    def __init__(self):
        self._bufs = {}

    def get(self, device, nbytes: int) -> torch.Tensor:
        key = (str(device), torch.cuda.current_stream(device).cuda_stream)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf


_WS = Workspace()


def workspace_size(T, k, H, I, E, has_shared) -> int:
    return int(L.lib().wmoe_workspace_size(T, k, H, I, E, int(has_shared)))


# --------------------------------------------------------------------------
# native expert forward
# --------------------------------------------------------------------------

def _mx_args(w13, s13, w2, s2):
    E, rows13, hb = w13.shape
    I = rows13 // 2
    H = hb * 2
    if s13.shape != (E, 2 * I, H // 32) or w2.shape != (E, H, I // 2) or s2.shape != (E, H, I // 32):
        raise ValueError("MXFP4 expert tensors have inconsistent shapes")
    for t in (w13, s13, w2, s2):
        if t.dtype != torch.uint8:
            raise ValueError("MXFP4 expert tensors must be uint8")
    return E, H, I


def experts_forward(x, indices, experts, *, order=None, swiglu_limit: float = 0.0, weights=None,
                    shared_expert: int = -1, shared_w=None, out=None, workspace=None, expert_range=None,
                    shared_rows=None, placement=None):
    """Grouped expert FFN on the device.

    ``weights is None``  -> un-reduced [..., k, H] (switch_mlp semantics);
    otherwise            -> [..., H] = sum_j w_j FFN_{idx_j}(x) (+ shared).
    ``experts``: BatchedExperts / QwenBatchedExperts (MXFP4) or Affine4BatchedExperts.

    ``expert_range=(base, count, n_routed)`` (MXFP4, with weights): one
    expert-parallel rank's share -- ``experts`` holds global routed experts
    [base, base+count) as local 0..count-1 (then the shared expert), other
    global ids are skipped, the shared expert runs only for rows in
    ``shared_rows=(lo, hi)`` (default all), and the result is the float32
    partial sum [..., H] that a reduce over the ranks completes.  With
    ``placement`` (int32 [n_routed] on the device, a permutation) the rank
    owns the routed ids whose placement positions lie in [base, base+count)
    instead (``ep.balanced_placement``).
    """
    if x.dtype != torch.bfloat16:
        raise ValueError("expert input must be bf16")
    H = x.shape[-1]
    k = indices.shape[-1]
    xf = x.reshape(-1, H).contiguous()
    T = xf.shape[0]
    idx = indices.reshape(-1, k).to(torch.int32).contiguous()
    if idx.shape[0] != T:
        raise ValueError("indices do not match the tokens")
    dev = x.device
    reduce = weights is not None
    if isinstance(experts, Affine4BatchedExperts):
        fmt = "affine4"
        E, rows13, hw = experts.w13.shape
        I = rows13 // 2
        if hw * 8 != H:
            raise ValueError("affine4 experts do not match the hidden size")
        order = experts.order if order is None else order
    else:
        fmt = "mxfp4"
        if isinstance(experts, QwenBatchedExperts):
            w13, s13, w2, s2 = experts.gate_up, experts.gate_up_scales, experts.down, experts.down_scales
            order = GATE_UP if order is None else order
        else:
            w13, s13, _ = experts.fused()
            w2, s2 = experts.w2, experts.w2_scales
            order = UP_GATE if order is None else order
        E, He, I = _mx_args(w13, s13, w2, s2)
        if He != H:
            raise ValueError("experts do not match the hidden size")
    has_shared = shared_expert is not None and shared_expert >= 0
    nbytes = workspace_size(T, k, H, I, E, has_shared)
    ws = workspace if workspace is not None else _WS.get(dev, nbytes)
    wts = weights.reshape(-1, k).float().contiguous() if reduce else None
    sw = shared_w.reshape(-1).float().contiguous() if shared_w is not None else None
    st = L.stream_of(xf)
    if expert_range is not None:
        if fmt != "mxfp4" or not reduce:
            raise ValueError("expert_range needs MXFP4 experts and routing weights")
        base, count, n_routed = (int(v) for v in expert_range)
        lo, hi = (0, T) if shared_rows is None else (int(shared_rows[0]), int(shared_rows[1]))
        if out is None:
            out = torch.empty((T, H), dtype=torch.float32, device=dev)
        if placement is not None and (placement.dtype != torch.int32 or placement.numel() != n_routed):
            raise ValueError("placement must be int32 [n_routed]")
        L.require_cuda(xf, idx, w13, s13, w2, s2, out, wts, sw, placement)
        L.call("wmoe_mxfp4_moe_forward_ep", L.ptr(xf), L.ptr(idx), L.ptr(wts), T, k, H, I, E, n_routed, base, count,
               L.ptr(placement), L.ptr(w13), L.ptr(s13), L.ptr(w2), L.ptr(s2), order, float(swiglu_limit),
               shared_expert if has_shared else -1, L.ptr(sw), lo, hi, L.ptr(out), L.ptr(ws), ws.numel(), st)
        return out.reshape(*x.shape[:-1], H)
    if out is None:
        out = torch.empty((T, H) if reduce else (T, k, H), dtype=torch.bfloat16, device=dev)
    if fmt == "mxfp4":
        L.require_cuda(xf, idx, w13, s13, w2, s2, out, wts, sw)
        if reduce:
            L.call("wmoe_mxfp4_moe_forward", L.ptr(xf), L.ptr(idx), L.ptr(wts), T, k, H, I, E, L.ptr(w13), L.ptr(s13),
                   L.ptr(w2), L.ptr(s2), order, float(swiglu_limit), shared_expert if has_shared else -1, L.ptr(sw),
                   L.ptr(out), L.ptr(ws), ws.numel(), st)
        else:
            L.call("wmoe_mxfp4_experts", L.ptr(xf), L.ptr(idx), T, k, H, I, E, L.ptr(w13), L.ptr(s13), L.ptr(w2),
                   L.ptr(s2), order, float(swiglu_limit), L.ptr(out), L.ptr(ws), ws.numel(), st)
    else:
        a = experts
        L.require_cuda(xf, idx, a.w13, a.w13_scales, a.w13_biases, a.w2, a.w2_scales, a.w2_biases, out, wts, sw)
        if reduce:
            L.call("wmoe_affine4_moe_forward", L.ptr(xf), L.ptr(idx), L.ptr(wts), T, k, H, I, E, L.ptr(a.w13),
                   L.ptr(a.w13_scales), L.ptr(a.w13_biases), L.ptr(a.w2), L.ptr(a.w2_scales), L.ptr(a.w2_biases),
                   a.group, order, float(swiglu_limit), shared_expert if has_shared else -1, L.ptr(sw), L.ptr(out),
                   L.ptr(ws), ws.numel(), st)
        else:
            L.call("wmoe_affine4_experts", L.ptr(xf), L.ptr(idx), T, k, H, I, E, L.ptr(a.w13), L.ptr(a.w13_scales),
                   L.ptr(a.w13_biases), L.ptr(a.w2), L.ptr(a.w2_scales), L.ptr(a.w2_biases), a.group, order,
                   float(swiglu_limit), L.ptr(out), L.ptr(ws), ws.numel(), st)
    lead = x.shape[:-1]
    return out.reshape(*lead, H) if reduce else out.reshape(*lead, k, H)


def permute(indices: torch.Tensor, num_experts: int):
    """Stable sort of the assignments by expert (mlx-lm _gather_sort semantics):
    (offsets [E+1], perm [T*k], inv [T*k]) int32."""
    idx = indices.reshape(indices.shape[0] if indices.dim() > 1 else 1, -1).to(torch.int32).contiguous()
    T, k = idx.shape
    L.require_cuda(idx)
    dev = idx.device
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    perm = torch.empty(T * k, dtype=torch.int32, device=dev)
    inv = torch.empty(T * k, dtype=torch.int32, device=dev)
    L.call("wmoe_permute", L.ptr(idx), T, k, num_experts, L.ptr(offsets), L.ptr(perm), L.ptr(inv), L.stream_of(idx))
    return offsets, perm, inv


class ClampedSwiGLU:
    """deepseek_v41/moe.py:30-43: the limit the expert kernel applies in its epilogue."""

    def __init__(self, limit: float = 0.0):
        self.limit = float(limit)


class StreamingSwitchGLU:
    """_StreamingSwitchGLU (model.py:276-459): ``switch(x, indices) -> [..., k, H]``.

    Experts come from ``cache.current_batched(layer)`` (HBM-resident); the
    sort-by-expert, both projections, the activation and the unsort run in
    the native expert path; ``record_gather_qmm`` is reported as the
    reference does (2 calls with a fused w13, else 3)."""

    def __init__(self, layer: int, cache, activation: ClampedSwiGLU | None = None):
        self.layer = layer
        self.cache = cache
        self.activation = activation or ClampedSwiGLU(0.0)

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        batched = self.cache.current_batched(self.layer)
        if batched is None:
            raise ValueError(f"layer {self.layer} has no resident experts")
        out = experts_forward(x, indices, batched, swiglu_limit=self.activation.limit)
        record = getattr(self.cache, "record_gather_qmm", None)
        if callable(record):
            calls = 2 if isinstance(batched, (QwenBatchedExperts, Affine4BatchedExperts)) or batched.w13 is not None else 3
            record(calls)
        return out


class StreamingExperts(StreamingSwitchGLU):
    """Qwen StreamingExperts (qwen4_exp.py:600-678): gate_up = [gate; up], plain SwiGLU."""

    def __init__(self, layer: int, cache):
        super().__init__(layer, cache, ClampedSwiGLU(0.0))
        self.grouped_prefill = True
