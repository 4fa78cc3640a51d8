"""The BASELINE configurations' synthetic layers, built on the host.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): this is what the timed
CPU restatement (``bench.py --impl reference`` and the ``cpu_baseline`` leg)
runs on, so that arm never loads the device library.  Shapes and
distributions are those of the device workloads (``whallm_b200.synthetic``);
the random draws come from host generators, so the values differ from the
device arm's while their statistics are the same:

  ds    -- H 7168, I 2048, 256 routed experts + 1 shared, top-8; expert
           weights N(0, 0.02) -> bf16 -> MXFP4 (Swift rule); gate rows
           N(0, 1/H) in bf16 (logits ~ N(0, 1)) plus a per-expert logit bias
           ln p_e, p_e ~ 1/rank^1.0 over a seeded permutation of the ranks;
           V4.1 gate (sqrt-softplus, eps 1e-20, route scale 1.5),
           ClampedSwiGLU(10).
  qn    -- H 2048, I 512, 512 + 1 shared, top-10, Zipf 1.1, the bf16 Qwen
           gate, shared expert gated by sigmoid(x . w_sg).
  tiny  -- H 1024, I 512, 16 experts, top-4, affine-4 group 64, router
           N(0, 0.02), the bf16 gate.

Experts are generated on first use: a CPU run builds only the experts its
tokens are routed to.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import build as _build
from . import formats as F
from . import moe as M
from . import router as R

CONFIGS = {
    "tiny": dict(H=1024, I=512, E=16, k=4, shared=False, zipf=None),
    "ds": dict(H=7168, I=2048, E=256, k=8, shared=True, zipf=1.0),
    "qn": dict(H=2048, I=512, E=512, k=10, shared=True, zipf=1.1),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(_build.build())
        _lib.oracle_normal_bf16.restype = None
        _lib.oracle_normal_bf16.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int64, ctypes.c_float,
                                            ctypes.c_void_p]
        _lib.oracle_mxfp4_quantize.restype = None
        _lib.oracle_mxfp4_quantize.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_void_p]
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def normal_bf16(seed: int, stream: int, shape, std: float) -> np.ndarray:
    """N(0, std) rounded to bf16 values (float32 array), counter-based and seeded."""
    out = np.empty(shape, np.float32)
    lib().oracle_normal_bf16(seed, stream, out.size, std, _p(out))
    return out


def mxfp4_quantize(vals: np.ndarray):
    """The Swift MXFP4 rule (same bytes as ``formats.mxfp4_quantize_values``), OpenMP in C."""
    v = np.ascontiguousarray(vals, np.float32)
    rows, cols = v.shape
    if cols % 32:
        raise ValueError("MXFP4 source must contain complete 32-value groups")
    packed = np.empty((rows, cols // 2), np.uint8)
    scales = np.empty((rows, cols // 32), np.uint8)
    lib().oracle_mxfp4_quantize(_p(v), rows, cols, _p(packed), _p(scales))
    return packed, scales


def zipf_logit_bias(E: int, alpha: float, seed: int) -> np.ndarray:
    """b_e = ln p_e, p_e proportional to 1/rank_e^alpha, ranks a seeded permutation of 1..E."""
    rank = np.random.default_rng(seed).permutation(E).astype(np.float64) + 1.0
    p = rank ** -alpha
    return np.log(p / p.sum()).astype(np.float32)


class _LazyExperts:
    """[E, ...] expert tensors whose rows are generated on first access."""

    def __init__(self, build):
        self._build = build
        self._cache = {}

    def get(self, e: int):
        if e not in self._cache:
            self._cache[e] = self._build(e)
        return self._cache[e]

    def __len__(self):
        return len(self._cache)


class _Field:
    def __init__(self, lazy, i):
        self.lazy, self.i = lazy, i

    def __getitem__(self, e):
        return self.lazy.get(int(e))[self.i]


class HostLayer:
    """One synthetic layer on the host: router tensors (bf16 bits), and an
    oracle expert set (``oracle.moe`` experts object) built on demand."""

    def __init__(self, name: str, seed: int = 0):
        cfg = dict(CONFIGS[name])
        self.name, self.cfg, self.seed = name, cfg, seed
        H, I, E = cfg["H"], cfg["I"], cfg["E"]
        if name == "tiny":
            self.gate_bits = F.f32_to_bf16_bits(normal_bf16(seed, 1, (E, H), 0.02))
            self.logit_bias = None
            self.shared_bits = None
        else:
            self.gate_bits = F.f32_to_bf16_bits(normal_bf16(seed, 1, (E, H), 1.0 / np.sqrt(H)))
            self.logit_bias = zipf_logit_bias(E, cfg["zipf"], seed + 3)
            self.shared_bits = (F.f32_to_bf16_bits(normal_bf16(seed, 2, (H,), 1.0 / np.sqrt(H)))
                                if name == "qn" else None)
        lazy = _LazyExperts(self._build_expert)
        self._lazy = lazy
        if name == "tiny":
            self.experts = M.Affine4Experts(*(_Field(lazy, i) for i in range(6)), M.GATE_UP, 0.0, 64)
        else:
            self.experts = M.MXFP4Experts(*(_Field(lazy, i) for i in range(4)),
                                          M.UP_GATE if name == "ds" else M.GATE_UP, 10.0 if name == "ds" else 0.0)

    def _build_expert(self, e: int):
        H, I = self.cfg["H"], self.cfg["I"]
        up = normal_bf16(self.seed + 2, 2 * e + 16, (2 * I, H), 0.02)
        down = normal_bf16(self.seed + 2, 2 * e + 17, (H, I), 0.02)
        if self.name == "tiny":
            return F.affine4_quantize(up, 64) + F.affine4_quantize(down, 64)
        return mxfp4_quantize(up) + mxfp4_quantize(down)

    @property
    def experts_built(self) -> int:
        return len(self._lazy)

    def route(self, x_f32):
        """Oracle router on bf16 tokens: (idx [T,k], weights [T,k], shared_w [T] or None)."""
        xb = F.f32_to_bf16_bits(x_f32)
        k = self.cfg["k"]
        if self.name == "ds":
            _, idx, w, _ = R.route(xb, self.gate_bits, k, R.SCORE_SQRTSOFTPLUS, logit_bias=self.logit_bias,
                                   norm_eps=1e-20, route_scale=1.5)
            return idx, w, None
        _, idx, w, sh = R.route(xb, self.gate_bits, k, R.SCORE_SOFTMAX_BF16, logit_bias=self.logit_bias,
                                norm_eps=0.0, wg_shared_bits=self.shared_bits)
        return idx, w, sh

    def prepare(self, idx):
        """Build every expert that the routes `idx` (and the shared expert) need."""
        for e in np.unique(np.asarray(idx)):
            self._lazy.get(int(e))
        if self.cfg["shared"]:
            self._lazy.get(self.cfg["E"])

    def forward(self, x_f32, idx=None, w=None, sh=None):
        """The whole layer: router (unless routes are given), experts, combine, shared expert."""
        if idx is None:
            idx, w, sh = self.route(x_f32)
        return M.moe_forward(x_f32, idx, w, self.experts, shared_expert=self.cfg["E"] if self.cfg["shared"] else None,
                             shared_weight=sh)


def tokens(T: int, H: int, seed: int) -> np.ndarray:
    """T tokens ~ N(0, 1) as bf16 values (float32 array)."""
    return normal_bf16(seed, 7, (T, H), 1.0)
