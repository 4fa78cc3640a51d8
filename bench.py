"""Benchmark of the routed-expert MoE layer (BASELINE metric: MoE layer tok/s).

Default workload: DeepSeek-class layer, H 7168, I 2048,
256 routed experts + 1 shared, top-8, MXFP4 weights, decode.  One step is one
pass of the decode batch sweep B = 1, 4, 16, 64 (85 tokens, four MoE-layer
forwards: router + experts + weighted combine + shared expert).  Each step
uses a different layer's weights out of 8 resident layers (48 GB), so weights
never come from L2 between steps; inputs are already in HBM.

  value  tokens/s over the whole job (sum over ranks / max rank time)
  e2e    the same through the public API with pinned host buffers: H2D of the
         step's tokens and D2H of the layer outputs inside the timed region
         (decode: on two copy streams, each copy overlapping another batch's
         layer replay)
  roofline  the expert FFN call (wmoe_mxfp4_moe_forward: permute, token
         split, tcgen05 up-projection + SwiGLU, tcgen05 down-projection,
         combine; the two tcgen05 launches carry ~90% of its device time):
         algorithmic bytes (distinct experts x 23,396,352 B + activations) /
         its CUDA-event time, against the measured HBM copy bandwidth
  breakdown  per batch size (back-to-back calls, layers cycled): layer and
         expert-call time, distinct experts, HBM fraction; and, on the same
         resident DeepSeek-class layers or on Qwen-class layers built beside
         them, ds_prefill_4096 (4096 tokens through the
         layer; its tensor fraction is against the dense bf16 peak, the rate of
         the two-term e4m3 token operand the block-scaled MMAs run),
         qn_decode_1 / qn_decode_32 and qn_prefill_16384.
         `--no-extras` skips those.
Decode batches are replayed as CUDA graphs (one per layer and batch size),
prefill runs eagerly.
  cpu_baseline  the oracle's C restatement (OpenMP, all host threads) on a
         bounded sample of the same sweep, on a layer built on the host

Other workloads: --workload ds_prefill (4096 tokens), qn_decode (B 1 and 32),
qn_prefill (16384 tokens), tiny (64 tokens, affine-4), kv (FP8 KV quantize +
dequantize of 32768 x 8 x 61 rows of 576), kv_scores (MXFP8 cache scores),
qsa (Qwen QSA affine KV caches: one decode update_and_fetch of 8 sequences at
a 32768-token context over the 12 full-attention layers), linear (dense MXFP8
linear, K = N = 5120: decode rows 1, 4, 16; 4096 in the breakdown).

`--impl reference` times the reference's algorithm on the host cores: the
oracle's restatement (router, grouped expert matmuls that dequantize inside
the loop, weighted combine, shared expert) on a layer of the same
configuration built on the host from seeds (``oracle/synthetic.py``); the
device library is not loaded.  The MLX CPU backend the reference would use is
not installable here.  It prints the same JSON line with "impl", the same
`config`, and the number of steps it actually timed.

Multi-GPU (torchrun): the MoE workloads run expert-parallel (`whallm_b200.ep`):
each rank routes its own tokens (weak scaling); the routed experts are dealt to
the ranks by popularity, equal counts per rank (WM_EP_PLACEMENT=contiguous for
plain ranges); decode gathers every rank's tokens and returns partial sums over
peer memory (WM_EP_EXCHANGE=nccl for NCCL collectives), prefill moves token rows
to the owning rank and back through NCCL all-to-all; the shared expert is
replicated; value = all ranks' tokens / max rank time.  The default line's
breakdown adds ep_prefill_4096: 4096 tokens per rank through the all-to-all
form.  Other workloads run as independent replicas.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DS_EXPERT_BYTES = 3 * 7168 * 2048 // 2 + 3 * 7168 * 2048 // 32   # 23,396,352
QN_EXPERT_BYTES = 3 * 2048 * 512 // 2 + 3 * 2048 * 512 // 32     # 1,671,168
TINY_EXPERT_BYTES = 884736
SWEEP = (1, 4, 16, 64)

MOE_WORKLOADS = {"ds_decode": ("ds", SWEEP), "ds_prefill": ("ds", (4096,)), "qn_decode": ("qn", (1, 32)),
                 "qn_prefill": ("qn", (16384,)), "tiny": ("tiny", (64,))}
GRAPHED = ("ds_decode", "qn_decode", "tiny")
EP_WORKLOADS = ("ds_decode", "ds_prefill", "qn_decode", "qn_prefill")
SHAPES = {"ds": dict(H=7168, I=2048, E=256, k=8, shared=True),
          "qn": dict(H=2048, I=512, E=512, k=10, shared=True),
          "tiny": dict(H=1024, I=512, E=16, k=4, shared=False)}
EXPERT_BYTES = {"ds": DS_EXPERT_BYTES, "qn": QN_EXPERT_BYTES, "tiny": TINY_EXPERT_BYTES}
MODEL = {"ds": "DeepSeek-class routed-expert layer: H 7168, I 2048, 256 routed + 1 shared experts, top-8, "
               "MXFP4 (E2M1, E8M0 per 32), V4.1 gate with a Zipf 1.0 logit bias, ClampedSwiGLU 10",
         "qn": "Qwen-Next-class sparse MoE layer: H 2048, I 512, 512 routed + 1 shared experts, top-10, MXFP4, "
               "bf16 gate with a Zipf 1.1 logit bias, sigmoid-gated shared expert",
         "tiny": "tiny MoE layer: H 1024, I 512, 16 experts, top-4, MLX affine 4-bit group 64, bf16 gate, "
                 "no shared expert"}
# bounded host samples of each MoE workload for the CPU restatement
CPU_SAMPLE = {"ds_decode": SWEEP, "ds_prefill": (256,), "qn_decode": (1, 32), "qn_prefill": (1024,), "tiny": (64,)}
REF_BUDGET_S = 150.0      # timed seconds of the reference arm (steps beyond it are not run, and not reported)
BASELINE_BUDGET_S = 25.0  # timed seconds of the cpu_baseline leg of our arm


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def _n_layers(args, name):
    return max(args.layers, 12) if name == "tiny" else args.layers     # 14.2 MB per tiny layer: 12 exceed L2


def _ep(args, world):
    return world > 1 and args.workload in EP_WORKLOADS


def workload_config(args, world):
    """The workload's description, printed identically by both arms."""
    wl = args.workload
    par = "single GPU" if world == 1 else "replicas"
    if wl in MOE_WORKLOADS:
        name, batches = MOE_WORKLOADS[wl]
        c = SHAPES[name]
        nl = _n_layers(args, name)
        n_exp = (args.experts or c["E"]) + (1 if c["shared"] else 0)
        cfg = {"workload": wl, "model": MODEL[name], "batches": list(batches), "tokens_per_step": sum(batches),
               "layers_cycled": nl,
               "l2": f"{nl} resident layers ({nl * n_exp * EXPERT_BYTES[name] / 1e9:.2f} GB of experts) cycled per "
                     "step: weights larger than L2"}
        if args.experts:
            cfg["routed_experts"] = args.experts
        if _ep(args, world):
            decode = wl in ("ds_decode", "qn_decode")
            peer = decode and os.environ.get("WM_EP_EXCHANGE", "peer") != "nccl"
            balanced = os.environ.get("WM_EP_PLACEMENT", "balanced") != "contiguous"
            cfg.update(parallelism=f"ep{world}", tokens_per_rank=sum(batches), experts_per_rank=c["E"] // world,
                       placement="popularity-balanced (snake order by router bias)" if balanced else "contiguous",
                       launch=("CUDA graph per (layer, batch): peer-memory exchange (CUDA IPC, flags), partial "
                               "experts" if peer else "CUDA graph per (layer, batch): NCCL all-gather, partial "
                               "experts, reduce-scatter") if decode else "eager (NCCL all-to-all)")
        else:
            cfg.update(parallelism=par, launch="CUDA graph per (layer, batch)" if wl in GRAPHED else "eager")
        return cfg
    if wl == "kv":
        return {"workload": wl, "rows_per_step": 32768 * 8 * args.kv_layers, "D": 576,
                "format": "e4m3 with one fp32 scale (amax/448) per 64 values", "sequences": 8, "context": 32768,
                "layers": args.kv_layers, "step": "quantize every row, then dequantize every row, layer by layer",
                "l2": "each layer's rows (302 MB bf16) exceed L2", "parallelism": par, "launch": "eager"}
    if wl == "kv_scores":
        return {"workload": wl, "sequences": 8, "context": 32768, "D": 512, "layers": args.kv_layers,
                "format": "MXFP8 (e4m3, E8M0 per 32)", "queries_per_sequence": 1,
                "l2": f"{args.kv_layers} layers of 145 MB caches: larger than L2", "parallelism": par,
                "launch": "eager"}
    if wl == "qsa":
        return {"workload": wl, "sequences": 8, "context": args.context, "full_attention_layers": 12,
                "caches": "K/V 8-bit 2 heads x 256, index 4-bit 1 head x 128, group 32",
                "step": "append one row per sequence + fetch the whole history, every cache",
                "l2": "the packed history read per step exceeds L2", "parallelism": par, "launch": "eager"}
    if wl == "linear":
        return {"workload": wl, "K": 5120, "N": 5120, "rows_per_step": [1, 4, 16], "weight_matrices_cycled": 8,
                "l2": "8 x 27 MB of weights cycled: larger than L2", "parallelism": par,
                "launch": "one CUDA graph per step (its three calls); the 4096-row calls eager"}
    raise SystemExit(f"unknown workload {wl}")


def workload_dtype(wl):
    if wl == "tiny":
        return "affine 4-bit weights (bf16 scale/bias per 64), bf16 activations, fp32 accumulate"
    if wl in MOE_WORKLOADS:
        return "mxfp4 weights, bf16 activations, fp32 accumulate"
    return {"kv": "e4m3 payload with fp32 scales, bf16 rows", "kv_scores": "e4m3 cache with E8M0 per 32, bf16 query",
            "qsa": "u32 packed affine 8/4-bit, bf16 scales/biases, bf16 out",
            "linear": "e4m3 weights with E8M0 per 32, bf16 activations, fp32 accumulate"}[wl]


def workload_data(wl):
    if wl in MOE_WORKLOADS:
        return ("synthetic (seeded N(0,0.02) expert weights quantized to the configuration's format, N(0,1) bf16 "
                "tokens, Zipf-skewed router)" if wl != "tiny" else
                "synthetic (seeded N(0,0.02) weights quantized to affine 4-bit, N(0,0.02) router, N(0,1) bf16 tokens)")
    return {"kv": "synthetic (seeded N(0,1) bf16 rows)", "kv_scores": "synthetic (seeded N(0,1) cache and query)",
            "qsa": "synthetic (seeded N(0,1) bf16 keys/values)",
            "linear": "synthetic (seeded N(0,0.02) weights quantized to MXFP8, N(0,1) bf16 rows)"}[wl]


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------
# workloads (our implementation)
# --------------------------------------------------------------------------

def _events(torch):
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def _e2e_overlapped(torch, dev, caps, hx, houts, steps):
    """ms per step of the decode sweep through captured layers with host I/O.

    caps[layer][batch] are CapturedLayer graphs; step i replays layer i % len(caps)
    for every batch.  The token batches go up from pinned host memory on one copy
    stream, straight into the graphs' inputs, and the outputs come down on
    another, so copies overlap the layer replays.  A layer's graphs are reused
    every len(caps) steps; their buffers are staged and replayed again only
    after the previous use's output copies are done, and every output copy is
    inside the timed region."""
    n_layers = len(caps)
    main = torch.cuda.current_stream(dev)
    cs_in, cs_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in hx]
    ev_g = [torch.cuda.Event() for _ in hx]
    layer_free = [torch.cuda.Event() for _ in range(n_layers)]
    for ev in layer_free:
        ev.record(main)
    s4, e4 = _events(torch)
    s4.record()
    for i in range(steps):
        li = i % n_layers
        cs_in.wait_event(layer_free[li])
        with torch.cuda.stream(cs_in):
            for b in range(len(hx)):
                caps[li][b].stage(hx[b])
                ev_in[b].record(cs_in)
        main.wait_event(layer_free[li])
        for b in range(len(hx)):
            main.wait_event(ev_in[b])
            y = caps[li][b].replay()
            ev_g[b].record(main)
            cs_out.wait_event(ev_g[b])
            with torch.cuda.stream(cs_out):
                houts[b].copy_(y, non_blocking=True)
        layer_free[li].record(cs_out)
    main.wait_stream(cs_out)
    e4.record()
    torch.cuda.synchronize()
    return s4.elapsed_time(e4) / steps


def _layer_launches(name, cfg, T):
    """Kernel launches of one layer forward, following the library's dispatch
    (csrc/moe_gemv.cu `run`): 2 router launches, then for the MXFP4 experts a
    permute unless the call has at most 64 (token, expert) slots (the first
    expert kernel groups them itself), the CUDA-core weight stream (up, down)
    for one- and two-token calls on experts with H <= 4096 and I <= 1024, else
    the token split and the two tcgen05 projections (plus the SwiGLU split in
    the prefill configuration), and the combine unless the call has at most
    64 slots and either takes the weight stream (each CTA of its down
    projection combines its own output rows) or has at most 4096 output values
    (the down projection's last CTA combines).
    Affine-4 (tiny): permute (unless at most 64 slots), f16 gather, two
    tcgen05 projections, combine."""
    if name == "tiny":
        return 2 + (4 if T * cfg["k"] <= 64 else 5)       # at most 64 slots: no permute launch
    H, I, k = cfg["H"], cfg["I"], cfg["k"]
    kk = k + (1 if cfg["shared"] else 0)
    S = T * kk
    n_routed = cfg["E"]
    stream = T <= 2 and H <= 4096 and I <= 1024
    small = S <= 64
    n = 2 + (0 if small else 1) + (0 if small and (stream or T * H <= 4096) else 1)
    if stream:
        n += 2
    else:
        decode = (T * k) // n_routed <= 32         # mx_tile_n: the decode configuration fuses the SwiGLU split
        n += 3 + (0 if decode else 1)
    return n


class MoeBench:
    """One MoE workload on resident synthetic layers: the routes of every
    (layer, batch), the distinct experts each reads (for the algorithmic byte
    count), CUDA graphs for decode shapes, and CUDA-event timing helpers.

    `layers` reuses already-built layers (another batch shape on the same
    weights); otherwise `n_layers` layers are built with per-rank seeds."""

    def __init__(self, torch, name, batches, graphed, dev, rank, n_layers=None, layers=None, experts=None):
        import whallm_b200 as W
        from whallm_b200 import experts as X
        from whallm_b200 import synthetic as S
        from whallm_b200.graphs import CapturedLayer
        self.torch, self.X = torch, X
        self.name, self.batches, self.graphed = name, tuple(batches), graphed
        self.layers = (layers if layers is not None else
                       [S.make_layer(name, dev, seed=1000 * rank + 17 * i, E=experts) for i in range(n_layers)])
        self.n_layers = len(self.layers)
        cfg = self.layers[0].cfg
        self.cfg = cfg
        self.xs = [S.make_tokens(B, cfg["H"], 100 + rank, dev) for B in self.batches]
        self.distinct = [0.0] * len(self.xs)
        self.routes = []
        for lay in self.layers:
            row = []
            for b, x in enumerate(self.xs):
                if name == "ds":
                    w, idx = lay.layer.gate(x)
                    sw = None
                else:
                    w, idx, sw = W.qwen_route(x, lay.gate_weight, cfg["k"], True, shared_gate=lay.shared_gate,
                                              logit_bias=lay.logit_bias)
                row.append((w, idx, sw))
                self.distinct[b] += (len(set(idx.flatten().tolist())) + (1 if cfg["shared"] else 0)) / self.n_layers
            self.routes.append(row)
        self.act_bytes = [x.numel() * 2 * 2 for x in self.xs]           # x in + out (bf16)
        self.alg_bytes = [d * EXPERT_BYTES[name] + a for d, a in zip(self.distinct, self.act_bytes)]
        kk = cfg["k"] + (1 if cfg["shared"] else 0)
        self.flops = [B * kk * 6 * cfg["H"] * cfg["I"] for B in self.batches]
        self.limit = 10.0 if name == "ds" else 0.0
        self.shared_id = cfg["E"] if cfg["shared"] else -1
        if graphed:
            self.caps = [[CapturedLayer(lay.layer, x) for x in self.xs] for lay in self.layers]
            self.ecaps = [[CapturedLayer(lambda xx, li=li, b=b: self.experts_call(li, b, xx), x)
                           for b, x in enumerate(self.xs)] for li in range(self.n_layers)]

    def experts_call(self, li, b, x):
        w, idx, sw = self.routes[li][b]
        return self.X.experts_forward(x, idx, self.layers[li].experts, weights=w, shared_expert=self.shared_id,
                                      shared_w=sw, swiglu_limit=self.limit)

    def layer(self, i, b):
        if self.graphed:
            return self.caps[i % self.n_layers][b]()
        return self.layers[i % self.n_layers].layer(self.xs[b])

    def experts(self, i, b):
        if self.graphed:
            return self.ecaps[i % self.n_layers][b]()
        return self.experts_call(i % self.n_layers, b, self.xs[b])

    def step(self, i):
        for b in range(len(self.xs)):
            self.layer(i, b)

    def experts_step(self, i):
        for b in range(len(self.xs)):
            self.experts(i, b)

    def timed(self, fn, reps):
        torch = self.torch
        torch.cuda.synchronize()
        s, e = _events(torch)
        s.record()
        for i in range(reps):
            fn(i)
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / reps

    def breakdown(self, reps, hbm, tc, prefix=""):
        """Per batch size: the whole layer and the expert call alone, back to back
        (layers cycled as in the timed step); hbm_frac = the expert call's
        algorithmic bytes over its time; prefill shapes add the tensor rate."""
        out = {}
        for b, B in enumerate(self.batches):
            t_layer = self.timed(lambda i, b=b: self.layer(i, b), reps)
            t_exp = self.timed(lambda i, b=b: self.experts(i, b), reps)
            d = {"ms": round(t_layer, 4), "tok_s": round(B / t_layer * 1e3, 1), "expert_ms": round(t_exp, 4),
                 "distinct_experts": round(self.distinct[b], 2),
                 "hbm_frac": round(self.alg_bytes[b] / (t_exp * 1e-3) / (hbm * 1e9), 4)}
            if B >= 1024:
                tf = self.flops[b] / (t_exp * 1e-3) / 1e12
                d["tflops"] = round(tf, 1)
                d["tensor_frac_bf16"] = round(tf / tc, 4)
            out[f"{prefix}{B}"] = d
        return out


def _moe_extras(torch, mb, args, dev, rank, hbm, tc, reps):
    """Breakdown entries of the default line beyond the decode sweep: the
    DeepSeek-class 4096-token prefill on the same layers, and the Qwen-class
    decode (B = 1, 32) and 16384-token prefill on Qwen-class layers."""
    out = {}
    pf = MoeBench(torch, "ds", (4096,), False, dev, rank, layers=mb.layers)
    pf.step(0)
    out.update(pf.breakdown(min(8, mb.n_layers), hbm, tc, prefix="ds_prefill_"))
    del pf
    qn = MoeBench(torch, "qn", (1, 32), True, dev, rank, n_layers=args.layers)
    for i in range(3):
        qn.step(i)
    out.update(qn.breakdown(reps, hbm, tc, prefix="qn_decode_"))
    qp = MoeBench(torch, "qn", (16384,), False, dev, rank, layers=qn.layers)
    qp.step(0)
    out.update(qp.breakdown(min(8, qn.n_layers), hbm, tc, prefix="qn_prefill_"))
    del qp, qn
    torch.cuda.empty_cache()
    return out


def run_ours(args, rank, world, dev):
    import torch
    import whallm_b200 as W
    from whallm_b200 import synthetic as S
    from whallm_b200.graphs import CapturedLayer

    torch.cuda.set_device(dev)
    hbm, tc, peak_src = _peaks()
    wl = args.workload
    res = {"hbm": hbm, "tc": tc, "peak_src": peak_src}
    if wl in MOE_WORKLOADS:
        name, batches = MOE_WORKLOADS[wl]
        mb = MoeBench(torch, name, batches, wl in GRAPHED, dev, rank, n_layers=_n_layers(args, name),
                      experts=args.experts)
        for i in range(args.warmup):
            mb.step(i)
        torch.cuda.synchronize()
        # timed region: whole MoE layer (router + experts + combine)
        clk = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
        if clk:
            clk.start()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        s, e = _events(torch)
        torch.cuda.nvtx.range_push("timed")
        s.record()
        for i in range(args.steps):
            mb.step(i)
        e.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.steps
        # expert-call roofline: the expert calls alone, same stream
        ms_exp = mb.timed(mb.experts_step, args.steps)
        clocks = clk.stop() if clk else None
        reps = max(2 * mb.n_layers, min(args.steps, 64))
        bd = mb.breakdown(reps, hbm, tc)
        # e2e through the public API with host buffers
        hx = [x.cpu().pin_memory() for x in mb.xs]
        houts = [torch.empty(x.shape, dtype=torch.bfloat16).pin_memory() for x in mb.xs]
        torch.cuda.synchronize()
        if mb.graphed:
            ms_e2e = _e2e_overlapped(torch, dev, mb.caps, hx, houts, args.steps)
        else:
            s4, e4 = _events(torch)
            s4.record()
            for i in range(args.steps):
                lay = mb.layers[i % mb.n_layers]
                for b in range(len(hx)):
                    houts[b].copy_(lay.layer(hx[b].to(dev, non_blocking=True)), non_blocking=True)
            e4.record()
            torch.cuda.synchronize()
            ms_e2e = s4.elapsed_time(e4) / args.steps
        if wl == "ds_decode" and not args.no_extras and args.experts is None:
            bd.update(_moe_extras(torch, mb, args, dev, rank, hbm, tc, reps))
        h2d = sum(x.numel() * 2 for x in mb.xs)
        prefill = wl in ("ds_prefill", "qn_prefill")
        res.update(dict(ms=ms, ms_exp=ms_exp, ms_e2e=ms_e2e, tokens=sum(batches), alg_bytes=sum(mb.alg_bytes),
                        flops=sum(mb.flops), prefill=prefill, breakdown=bd, clocks=clocks, h2d=h2d, d2h=h2d,
                        distinct=mb.distinct,
                        launches=sum(_layer_launches(name, mb.cfg, B) for B in mb.batches),
                        kernel="expert FFN call (wmoe_mxfp4_moe_forward)" if name != "tiny"
                        else "expert FFN call (wmoe_affine4_moe_forward)"))
        return res
    if wl == "kv_scores":
        # decode scores of one query per sequence against an MXFP8 latent cache:
        # 8 sequences x 32768 cached tokens x 512 dims per layer, kv_layers layers (each its own cache)
        Bq, Lc, D, n_layer = 8, 32768, 512, args.kv_layers
        caches = []
        for li in range(n_layer):
            kvr = torch.randn(Bq * Lc, D, device=dev, generator=torch.Generator(device=dev).manual_seed(li))
            pl, sc = W.kv_quantize(kvr.to(torch.bfloat16), "mxfp8")
            caches.append((pl.view(Bq, Lc, D), sc.view(Bq, Lc, D // 32)))
            del kvr
        q = torch.randn(Bq, 1, D, device=dev).to(torch.bfloat16)
        out = torch.empty(Bq, 1, Lc, dtype=torch.bfloat16, device=dev)
        for i in range(args.warmup):
            W.kv_scores(q, *caches[i % n_layer], "mxfp8", out=out)
        torch.cuda.synchronize()
        clk = ClockSampler(dev.index if dev.index is not None else 0)
        clk.start()
        s, e = _events(torch)
        s.record()
        for _ in range(args.steps):
            for li in range(n_layer):
                W.kv_scores(q, *caches[li], "mxfp8", out=out)
        e.record()
        torch.cuda.synchronize()
        clocks = clk.stop()
        ms = s.elapsed_time(e) / args.steps
        per_layer = Bq * Lc * (D + D // 32) + Bq * D * 2 + Bq * Lc * 2
        hq = q.cpu().pin_memory()
        hout = torch.empty(out.shape, dtype=torch.bfloat16).pin_memory()
        torch.cuda.synchronize()
        s4, e4 = _events(torch)
        s4.record()
        for _ in range(args.steps):
            for li in range(n_layer):
                hout.copy_(W.kv_scores(hq.to(dev, non_blocking=True), *caches[li], "mxfp8", out=out),
                           non_blocking=True)
        e4.record()
        torch.cuda.synchronize()
        ms_e2e = s4.elapsed_time(e4) / args.steps
        res.update(dict(ms=ms, ms_exp=ms, ms_e2e=ms_e2e, tokens=Bq * Lc * n_layer, alg_bytes=per_layer * n_layer,
                        breakdown={}, clocks=clocks, flops=0, h2d=Bq * D * 2 * n_layer, d2h=Bq * Lc * 2 * n_layer,
                        launches=3 * n_layer,
                        kernel="KV-cache score launch (wkv_mx_scores: query split, tcgen05 block-scaled scores)"))
        return res
    if wl == "qsa":
        # Qwen QSA caches in decode: 12 full-attention layers, each an 8-bit K/V cache of
        # 2 kv heads x 256 and a 4-bit indexer cache of 1 head x 128; 8 sequences at a
        # 32768-token context; one step appends one token per sequence and fetches the
        # whole dequantized history of every cache (update_and_fetch)
        from whallm_b200.kvcache import QSAQuantizedCache
        Bq, Lc, n_layer = 8, args.context, 12
        shapes = ((8, 2, 256), (4, 1, 128))      # (bits, kv heads, head dim)
        cap = Lc + args.warmup + 2 * args.steps     # warm-up, timed and end-to-end steps each append a row
        caches = []
        for li in range(n_layer):
            pair = []
            for bits, hk, hd in shapes:
                c = QSAQuantizedCache(bits, hd, capacity=cap)
                g = torch.Generator(device=dev).manual_seed(li * 2 + bits)
                kx = torch.randn(Bq, hk, Lc - 1, hd, device=dev, generator=g).to(torch.bfloat16)
                c.update_and_fetch(kx, kx)
                pair.append(c)
            caches.append(pair)
            del kx
        torch.cuda.empty_cache()
        news = [torch.randn(Bq, hk, 1, hd, device=dev).to(torch.bfloat16) for _, hk, hd in shapes]

        def step(news_):
            outs = []
            for pair in caches:
                for c, x in zip(pair, news_):
                    outs.append(c.update_and_fetch(x, x))
            return outs

        for _ in range(args.warmup):
            step(news)
        torch.cuda.synchronize()
        clk = ClockSampler(dev.index if dev.index is not None else 0)
        clk.start()
        s, e = _events(torch)
        s.record()
        for _ in range(args.steps):
            step(news)
        e.record()
        torch.cuda.synchronize()
        clocks = clk.stop()
        ms = s.elapsed_time(e) / args.steps
        # the dominant kernel alone: the history fetch of every cache
        s2, e2 = _events(torch)
        s2.record()
        for _ in range(args.steps):
            for pair in caches:
                for c in pair:
                    c.fetch()
        e2.record()
        torch.cuda.synchronize()
        ms_exp = s2.elapsed_time(e2) / args.steps
        L_now = caches[0][0].offset
        rd = wr = 0
        for bits, hk, hd in shapes:   # per layer: K and V, packed + bf16 scale/bias read, bf16 written
            rd += 2 * Bq * hk * L_now * (hd * bits // 8 + 4 * (hd // 32)) * n_layer
            wr += 2 * Bq * hk * L_now * 2 * hd * n_layer
        alg = rd + wr
        # end to end: the new rows come from pinned host memory, the newest dequantized
        # row of every cache goes back
        hnews = [x.cpu().pin_memory() for x in news]
        hlast = [torch.empty((Bq, hk, hd), dtype=torch.bfloat16).pin_memory() for _, hk, hd in shapes]
        torch.cuda.synchronize()
        s4, e4 = _events(torch)
        s4.record()
        for _ in range(args.steps):
            dn = [x.to(dev, non_blocking=True) for x in hnews]
            outs = step(dn)
            for i, (ko, _vo) in enumerate(outs):
                hlast[i % 2].copy_(ko[:, :, -1], non_blocking=True)
        e4.record()
        torch.cuda.synchronize()
        ms_e2e = s4.elapsed_time(e4) / args.steps
        h2d = sum(x.numel() * 2 for x in hnews)
        d2h = n_layer * sum(Bq * hk * hd * 2 for _, hk, hd in shapes)
        res.update(dict(ms=ms, ms_exp=ms_exp, ms_e2e=ms_e2e, tokens=Bq * Lc * n_layer, alg_bytes=alg,
                        breakdown={"history_read_gb_per_step": round(rd / 1e9, 2),
                                   "bf16_written_gb_per_step": round(wr / 1e9, 2)},
                        clocks=clocks, flops=0, h2d=h2d, d2h=d2h, launches=4 * n_layer,
                        kernel="history fetch of every QSA cache (k_affine_kv_fetch, K and V in one launch)"))
        return res
    if wl == "linear":
        # dense MXFP8 linear (the QuantizedLinear layers V4.1 builds from its
        # native-FP8 attention and shared-expert weights): K 5120 -> N 5120;
        # one step = the decode rows T = 1, 4, 16, each call on another of 8
        # weight matrices (210 MB: weights come from HBM); T = 4096 is reported
        # in the breakdown against the tensor peak
        K = N = 5120
        sweep = (1, 4, 16)
        mats = []
        for li in range(8):
            g = torch.Generator(device=dev).manual_seed(li)
            w = torch.randn((N, K), generator=g, device=dev).mul_(0.02).to(torch.bfloat16)
            mats.append(W.MXFP8Linear.quantize(w))
            del w
        xs_l = [S.make_tokens(T, K, 7 + T, dev) for T in sweep]
        outs = [torch.empty((T, N), dtype=torch.bfloat16, device=dev) for T in sweep]

        def capture(calls):
            """One CUDA graph of several linear calls (j, matrix): a decode step replays
            its linears from one graph, so launches overlap their neighbours' tails
            (programmatic dependent launch) and the host's replay cost is paid once."""
            for j, li in calls:
                W.mx_linear(xs_l[j], mats[li].weight, mats[li].scales, "mxfp8", out=outs[j])
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for j, li in calls:
                    W.mx_linear(xs_l[j], mats[li].weight, mats[li].scales, "mxfp8", out=outs[j])
            return g

        # step i: the decode rows T = 1, 4, 16, each on another of the 8 matrices
        step_graphs = [capture([(j, (3 * i + j) % 8) for j in range(len(sweep))]) for i in range(8)]

        def lstep(i):
            step_graphs[i % 8].replay()

        for i in range(args.warmup):
            lstep(i)
        torch.cuda.synchronize()
        clk = ClockSampler(dev.index if dev.index is not None else 0)
        clk.start()
        s, e = _events(torch)
        torch.cuda.nvtx.range_push("timed")
        s.record()
        for i in range(args.steps):
            lstep(i)
        e.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        clocks = clk.stop()
        ms = s.elapsed_time(e) / args.steps
        wbytes = N * K + N * (K // 32)
        alg = sum(wbytes + T * K * 2 + T * N * 2 for T in sweep)
        per_b = {}
        for j, T in enumerate(sweep):
            g8 = capture([(j, li) for li in range(8)])      # the 8 matrices in turn, rows T
            g8.replay()
            torch.cuda.synchronize()
            s3, e3 = _events(torch)
            s3.record()
            for i in range(4):
                g8.replay()
            e3.record()
            torch.cuda.synchronize()
            t_ms = s3.elapsed_time(e3) / 32
            del g8
            per_b[str(T)] = {"ms": round(t_ms, 4), "hbm_frac": round((wbytes + T * K * 2 + T * N * 2) /
                                                                      (t_ms * 1e-3) / (hbm * 1e9), 4)}
        xp = S.make_tokens(4096, K, 11, dev)
        yp = torch.empty((4096, N), dtype=torch.bfloat16, device=dev)
        W.mx_linear(xp, mats[0].weight, mats[0].scales, "mxfp8", out=yp)
        torch.cuda.synchronize()
        s3, e3 = _events(torch)
        s3.record()
        for i in range(8):
            W.mx_linear(xp, mats[i].weight, mats[i].scales, "mxfp8", out=yp)
        e3.record()
        torch.cuda.synchronize()
        t_ms = s3.elapsed_time(e3) / 8
        per_b["4096"] = {"ms": round(t_ms, 4), "tflops": round(2 * 4096 * N * K / (t_ms * 1e-3) / 1e12, 1),
                         "tensor_frac": round(2 * 4096 * N * K / (t_ms * 1e-3) / (tc * 1e12), 4)}
        # end to end: rows from pinned host memory, outputs back
        hx = [x.cpu().pin_memory() for x in xs_l]
        ho = [torch.empty(o.shape, dtype=torch.bfloat16).pin_memory() for o in outs]
        torch.cuda.synchronize()
        s4, e4 = _events(torch)
        s4.record()
        for i in range(args.steps):
            for j in range(len(sweep)):
                xs_l[j].copy_(hx[j], non_blocking=True)
            lstep(i)
            for j in range(len(sweep)):
                ho[j].copy_(outs[j], non_blocking=True)
        e4.record()
        torch.cuda.synchronize()
        ms_e2e = s4.elapsed_time(e4) / args.steps
        res.update(dict(ms=ms, ms_exp=ms, ms_e2e=ms_e2e, tokens=sum(sweep), alg_bytes=alg, breakdown=per_b,
                        clocks=clocks, flops=0, h2d=sum(T * K * 2 for T in sweep), d2h=sum(T * N * 2 for T in sweep),
                        launches=1 + 3 * (len(sweep) - 1),
                        kernel="dense MXFP8 linear calls (wmx_linear: one row on the CUDA-core weight stream; "
                               "4 and 16 rows as token split, tcgen05 block-scaled GEMM split over K, ordered "
                               "sum of the K splits)"))
        return res
    if wl == "kv":
        # quantize every row of a 8 x 32768-token MLA cache (576 = 512 latent + 64 rope,
        # e4m3 with an fp32 scale per 64), then dequantize it, layer by layer
        D, rows_total = 576, 32768 * 8 * args.kv_layers
        chunk = 32768 * 8          # one layer of the 8 x 32768-token context per call
        x = torch.randn(chunk, D, device=dev).to(torch.bfloat16)
        p, sc = W.kv_quantize(x, "fp8_f32_b64")
        out = torch.empty_like(x)
        for _ in range(args.warmup):
            W.kv_quantize(x, "fp8_f32_b64", p, sc)
            W.kv_dequantize(p, sc, "fp8_f32_b64", out)
        torch.cuda.synchronize()
        clk = ClockSampler(dev.index if dev.index is not None else 0)
        clk.start()
        s, e = _events(torch)
        torch.cuda.nvtx.range_push("timed")
        s.record()
        for _ in range(args.steps):
            for _l in range(args.kv_layers):
                W.kv_quantize(x, "fp8_f32_b64", p, sc)
                W.kv_dequantize(p, sc, "fp8_f32_b64", out)
        e.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        clocks = clk.stop()
        ms = s.elapsed_time(e) / args.steps
        per_entry = 576 + 9 * 4 + 1152
        alg = rows_total * per_entry * 2  # quantize (read bf16, write packed) + dequant (read packed, write bf16)
        # the two kernels alone, for the breakdown
        tq = _events(torch)
        td = _events(torch)
        tq[0].record()
        for _l in range(args.kv_layers):
            W.kv_quantize(x, "fp8_f32_b64", p, sc)
        tq[1].record()
        td[0].record()
        for _l in range(args.kv_layers):
            W.kv_dequantize(p, sc, "fp8_f32_b64", out)
        td[1].record()
        torch.cuda.synchronize()
        half = chunk * per_entry * args.kv_layers
        bd = {"quantize": {"ms_per_layer": round(tq[0].elapsed_time(tq[1]) / args.kv_layers, 4),
                           "hbm_frac": round(half / (tq[0].elapsed_time(tq[1]) * 1e-3) / (hbm * 1e9), 4)},
              "dequantize": {"ms_per_layer": round(td[0].elapsed_time(td[1]) / args.kv_layers, 4),
                             "hbm_frac": round(half / (td[0].elapsed_time(td[1]) * 1e-3) / (hbm * 1e9), 4)}}
        # e2e: every layer's rows come up from pinned host memory and its dequantized rows go back, on two
        # copy streams overlapping the kernels of the neighbouring layers (double-buffered device rows)
        hx = x.cpu().pin_memory()
        hout = torch.empty_like(hx).pin_memory()
        dx = [torch.empty_like(x) for _ in range(2)]
        dout = [torch.empty_like(x) for _ in range(2)]
        main = torch.cuda.current_stream(dev)
        cs_in, cs_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_q = [torch.cuda.Event() for _ in range(2)]
        ev_c = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        for ev in ev_q + ev_out:
            ev.record(main)
        n_e2e = min(args.steps, 2)
        torch.cuda.synchronize()
        s4, e4 = _events(torch)
        s4.record()
        for j in range(n_e2e * args.kv_layers):
            b = j % 2
            cs_in.wait_event(ev_q[b])
            with torch.cuda.stream(cs_in):
                dx[b].copy_(hx, non_blocking=True)
                ev_in[b].record(cs_in)
            main.wait_event(ev_in[b])
            main.wait_event(ev_out[b])
            W.kv_quantize(dx[b], "fp8_f32_b64", p, sc)
            ev_q[b].record(main)
            W.kv_dequantize(p, sc, "fp8_f32_b64", dout[b])
            ev_c[b].record(main)
            cs_out.wait_event(ev_c[b])
            with torch.cuda.stream(cs_out):
                hout.copy_(dout[b], non_blocking=True)
                ev_out[b].record(cs_out)
        main.wait_stream(cs_out)
        e4.record()
        torch.cuda.synchronize()
        ms_e2e = s4.elapsed_time(e4) / n_e2e
        layer_bytes = chunk * D * 2
        res.update(dict(ms=ms, ms_exp=ms, ms_e2e=ms_e2e, tokens=rows_total, alg_bytes=alg, breakdown=bd,
                        clocks=clocks, flops=0, h2d=layer_bytes * args.kv_layers, d2h=layer_bytes * args.kv_layers,
                        launches=2 * args.kv_layers,
                        kernel="FP8 KV quantize + dequantize (k_kv_fp8_quantize, k_kv_fp8_dequantize)"))
        return res
    raise SystemExit(f"unknown workload {wl}")


def run_ep(args, rank, world, dev):
    """Expert-parallel layer over NCCL: the routed experts are sharded evenly
    (E/W per rank), the router and the shared expert are replicated.  Decode
    uses the gathered form (all-gather tokens and routes, partial sums of the
    rank's experts, reduce-scatter; fixed-size collectives, one CUDA graph per
    (layer, batch)); prefill uses the variable-split all-to-all form, eager."""
    import torch
    import whallm_b200 as W
    from whallm_b200 import ep as EP
    from whallm_b200 import synthetic as S
    from whallm_b200.graphs import CapturedLayer

    torch.cuda.set_device(dev)
    hbm, tc, peak_src = _peaks()
    wl = args.workload
    name, batches = MOE_WORKLOADS[wl]
    decode = wl in ("ds_decode", "qn_decode")
    # decode exchanges over peer memory (CUDA IPC + flags) unless WM_EP_EXCHANGE=nccl
    peer = decode and os.environ.get("WM_EP_EXCHANGE", "peer") != "nccl"
    n_layers = args.layers
    # experts dealt to the ranks by popularity (the router's per-expert bias),
    # unless WM_EP_PLACEMENT=contiguous
    balanced = os.environ.get("WM_EP_PLACEMENT", "balanced") != "contiguous"
    extras = wl == "ds_decode" and not args.no_extras
    moes = []
    prefill_moes = []                                       # the all-to-all form on the same shards (extras)
    owned = []                                              # per layer: this rank's routed expert ids
    cfg = None
    bufs = None
    for i in range(n_layers):
        lay = S.make_layer(name, dev, seed=17 * i)          # identical weights on every rank
        cfg = lay.cfg
        E = cfg["E"]
        e0, per = EP.shard_bounds(E, world, rank)
        order = EP.balanced_placement(lay.logit_bias.exp(), world) if balanced and lay.logit_bias is not None else None
        pos = EP.placement_positions(order, dev) if order is not None else None
        owned.append(set(order[e0:e0 + per].tolist()) if order is not None else set(range(e0, e0 + per)))
        local = EP.shard_experts(lay.experts, rank, world, E, cfg["shared"], order=order)
        limit = 10.0 if name == "ds" else 0.0
        if name == "ds":
            router = lay.layer.gate
            gate_fn = None
        else:
            state = {}

            def router(x, lay=lay, state=state):
                w, idx, sw = W.qwen_route(x, lay.gate_weight, cfg["k"], True, shared_gate=lay.shared_gate,
                                          logit_bias=lay.logit_bias)
                state["sw"] = sw
                return (w, idx, sw) if decode else (w, idx)

            def gate_fn(x, state=state):
                return state["sw"]
        if peer:
            if bufs is None:
                bufs = EP.PeerBuffers(max(batches), cfg["H"], cfg["k"], device=dev)
            moes.append([EP.PeerGatheredMoE(router, local, E, B, bufs, limit, cfg["shared"], shared_gated=name != "ds",
                                            positions=pos)
                         for B in batches])
        elif decode:
            moes.append(EP.GatheredExpertParallelMoE(
                router, EP.gpu_partial_experts(local, e0, per, E, limit, cfg["shared"], positions=pos), E))
        else:
            moes.append(EP.ExpertParallelMoE(router, EP.gpu_local_experts(local, limit), E,
                                             shared=EP.gpu_shared_expert(local, per, limit, gate=gate_fn),
                                             positions=pos))
        if extras and i < 4:
            prefill_moes.append(EP.ExpertParallelMoE(router, EP.gpu_local_experts(local, limit), E,
                                                     shared=EP.gpu_shared_expert(local, per, limit), positions=pos))
        if not peer:
            moes[-1].route_fn = router
        del lay
        torch.cuda.empty_cache()
    H = cfg["H"]
    xs = [S.make_tokens(B, H, 100 + rank, dev) for B in batches]
    # algorithmic bytes: the distinct local experts each (layer, batch) touches
    # over all ranks' tokens, plus the shared expert, plus activations
    expert_bytes = EXPERT_BYTES[name]
    distinct = [0.0] * len(xs)
    for m, mine in zip(moes, owned):
        for b, x in enumerate(xs):
            route_fn = m[b].router if isinstance(m, list) else m.route_fn
            idx = route_fn(x)[1].to(torch.int32).contiguous()
            allidx = torch.empty((world * idx.shape[0], idx.shape[1]), dtype=idx.dtype, device=dev)
            torch.distributed.all_gather_into_tensor(allidx, idx)
            ids = set(allidx.flatten().tolist())
            distinct[b] += (len(ids & mine) + (1 if cfg["shared"] else 0)) / n_layers
    act_bytes = sum(world * B * H * (2 + 4 + 4) for B in batches) if decode else 0
    alg_bytes = sum(distinct) * expert_bytes + act_bytes

    if decode:
        caps = [[CapturedLayer(m[b] if isinstance(m, list) else m, x) for b, x in enumerate(xs)] for m in moes]

        def call(li, b, x=None):
            return caps[li][b](x)
    else:
        def call(li, b, x=None):
            return moes[li](xs[b] if x is None else x)

    def step(i):
        for b in range(len(xs)):
            call(i % n_layers, b)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    clk = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if clk:
        clk.start()
    torch.distributed.barrier()
    torch.cuda.synchronize()
    s, e = _events(torch)
    s.record()
    for i in range(args.steps):
        step(i)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    clocks = clk.stop() if clk else None
    torch.distributed.barrier()
    hx = [x.cpu().pin_memory() for x in xs]
    houts = [torch.empty(x.shape, dtype=torch.bfloat16).pin_memory() for x in xs]
    torch.cuda.synchronize()
    if decode:
        ms_e2e = _e2e_overlapped(torch, dev, caps, hx, houts, args.steps)
    else:
        s4, e4 = _events(torch)
        s4.record()
        for i in range(args.steps):
            for b in range(len(xs)):
                houts[b].copy_(call(i % n_layers, b, hx[b].to(dev, non_blocking=True)), non_blocking=True)
        e4.record()
        torch.cuda.synchronize()
        ms_e2e = s4.elapsed_time(e4) / args.steps
    if decode:
        del caps           # graphs holding NCCL work go before the process group
        torch.cuda.synchronize()
    breakdown = {}
    if prefill_moes:
        # 4096 tokens per rank through the all-to-all form, max over ranks
        xp = S.make_tokens(4096, H, 200 + rank, dev)
        prefill_moes[0](xp)
        torch.cuda.synchronize()
        torch.distributed.barrier()
        s5, e5 = _events(torch)
        s5.record()
        reps = 2 * len(prefill_moes)
        for i in range(reps):
            prefill_moes[i % len(prefill_moes)](xp)
        e5.record()
        torch.cuda.synchronize()
        t = torch.tensor([s5.elapsed_time(e5) / reps], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        pms = float(t.item())
        breakdown["ep_prefill_4096"] = {"ms": round(pms, 4), "tok_s": round(world * 4096 / pms * 1e3, 1),
                                        "tokens_per_rank": 4096, "layers_cycled": len(prefill_moes),
                                        "launch": "eager (NCCL all-to-all)"}
        del xp
    prefill_moes.clear()
    if bufs is not None:
        bufs.check()
        del moes
        bufs.close()
    h2d = sum(x.numel() * 2 for x in xs)
    return dict(ms=ms, ms_exp=ms, ms_e2e=ms_e2e, tokens=sum(batches), alg_bytes=alg_bytes, breakdown=breakdown,
                clocks=clocks, h2d=h2d, d2h=h2d, distinct=distinct, hbm=hbm, tc=tc, peak_src=peak_src,
                launches=len(xs) * ((11 if peer else 7) if decode else 9), flops=0, ep=True, decode=decode,
                kernel="whole layer per rank (router, exchange, expert share)")


# --------------------------------------------------------------------------
# reference arm: the oracle restatement on the host cores
# --------------------------------------------------------------------------

def cpu_reference(args, steps, warmup, budget_s):
    """Times the oracle's restatement of the reference path on the host cores.

    MoE workloads: the reference MoE layer (router, grouped expert matmuls that
    dequantize inside the loop, weighted combine, shared expert) on a layer of
    the workload's configuration built on the host (``oracle/synthetic.py``:
    seeded weights, the Swift MXFP4 rule; only the experts the sample's tokens
    are routed to), over a bounded token sample (CPU_SAMPLE).  KV workloads:
    the numpy restatements of one layer's rows.  No device library is loaded.

    Runs `warmup` untimed steps (fewer if one step is slow), then times `steps`
    steps, or as many as fit in `budget_s` seconds; returns the counts run."""
    import numpy as np
    from oracle import formats as F

    threads = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    wl = args.workload
    if wl == "kv":
        D, n = 576, 32768
        x = F.round_bf16(np.random.default_rng(0).normal(0, 1, (n, D)).astype(np.float32))

        def step():
            p, s = F.kv_quantize(x, F.KV_FP8_F32_B64)
            F.kv_dequantize(p, s, F.KV_FP8_F32_B64, D)

        tokens, sample = n, "kv: 32768 rows of 576 (one sequence, one layer), numpy oracle"
    elif wl == "kv_scores":
        D, n = 512, 32768
        rng = np.random.default_rng(0)
        x = F.round_bf16(rng.normal(0, 1, (n, D)).astype(np.float32))
        p, s = F.kv_quantize(x, F.KV_MXFP8_B32)
        q = F.round_bf16(rng.normal(0, 1, (1, 1, D)).astype(np.float32))

        def step():
            F.kv_scores(q, p.reshape(1, n, -1), s.reshape(1, n, -1), F.KV_MXFP8_B32, D)

        tokens, sample = n, "kv_scores: one query against 32768 MXFP8 rows of 512 (one sequence, one layer), numpy oracle"
    elif wl == "linear":
        K = N = 5120
        rng = np.random.default_rng(0)
        w = F.round_bf16(rng.normal(0, 0.02, (N, K)).astype(np.float32))
        p, s = F.kv_quantize(w, F.KV_MXFP8_B32)
        q = F.round_bf16(rng.normal(0, 1, (1, 16, K)).astype(np.float32))

        def step():
            F.kv_scores(q, p.reshape(1, N, -1), s.reshape(1, N, -1), F.KV_MXFP8_B32, K)

        tokens, sample = 16, "linear: 16 rows through one MXFP8 [5120 x 5120] weight, numpy oracle (float64 product)"
    elif wl == "qsa":
        n = 32768
        rng = np.random.default_rng(0)
        caches = []
        for bits, hk, hd in ((8, 2, 256), (4, 1, 128)):
            c = F.QSACache(bits, hd)
            x = F.f32_to_bf16_bits(rng.normal(0, 1, (hk, n - 1, hd)).astype(np.float32))
            c.update_and_fetch(x, x)
            caches.append((c, F.f32_to_bf16_bits(rng.normal(0, 1, (hk, 1, hd)).astype(np.float32))))

        def step():
            for c, x in caches:
                c.update_and_fetch(x, x)

        tokens = n
        sample = ("qsa: one decode update_and_fetch of one sequence at a 32768-token context, one layer's two QSA "
                  "caches (8-bit 2x256 K/V, 4-bit 1x128 index), numpy oracle")
    else:
        from oracle import synthetic as SY
        name, _ = MOE_WORKLOADS[wl]
        batches = CPU_SAMPLE[wl]
        lay = SY.HostLayer(name, seed=0)
        H = lay.cfg["H"]
        xs = [SY.tokens(B, H, 100 + j) for j, B in enumerate(batches)]
        for x in xs:                                   # build the experts the sample is routed to
            lay.prepare(lay.route(x)[0])

        def step():
            for x in xs:
                lay.forward(x)                         # router + experts + combine + shared expert

        tokens = sum(batches)
        sample = (f"{wl}: batches {list(batches)} ({tokens} tokens per step) on a full-size layer built on the host "
                  f"({lay.experts_built} experts materialised); oracle router + C expert matmuls with in-loop "
                  f"dequant, {threads} threads")
    t0 = time.perf_counter()
    step()
    t_step = time.perf_counter() - t0
    warm = 1
    while warm < warmup and (warm + 1) * t_step < budget_s / 4:
        step()
        warm += 1
    n = steps if steps * t_step <= budget_s else max(1, int(budget_s / t_step))
    t0 = time.perf_counter()
    for _ in range(n):
        step()
    dt = (time.perf_counter() - t0) / n
    # the KV restatements are single-threaded numpy; the MoE arm runs the C kernels on every host thread
    cores = 1 if wl in ("kv", "kv_scores", "qsa", "linear") else threads
    return dict(value=tokens / dt, sec_per_step=dt, tokens=tokens, cores=cores, sample=sample, steps=n, warmup=warm)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="ds_decode",
                    choices=["ds_decode", "ds_prefill", "qn_decode", "qn_prefill", "tiny", "kv", "kv_scores", "qsa",
                             "linear"])
    ap.add_argument("--layers", type=int, default=8, help="resident layers cycled per step (no L2 reuse)")
    ap.add_argument("--experts", type=int, default=None,
                    help="routed experts per layer (default: the configuration's); smaller layers for ncu captures")
    ap.add_argument("--context", type=int, default=32768,
                    help="qsa workload: tokens already cached per sequence (smaller for ncu captures)")
    ap.add_argument("--kv-layers", type=int, default=61,
                    help="kv and kv_scores workloads: cache layers held on the device (61 in the configuration; "
                         "a few for ncu captures, which keep each layer's cache resident)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the breakdown's prefill and Qwen-class entries of the default workload")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    unit = {"kv": "KV rows/s", "kv_scores": "cached rows scored/s", "qsa": "context rows fetched/s",
            "linear": "rows/s"}.get(args.workload, "tokens/s")
    metric = {"ds_decode": "MoE layer tok/s, DeepSeek-class MXFP4 decode sweep B=1,4,16,64",
              "kv": "FP8 KV quantize+dequantize rows/s",
              "kv_scores": "MXFP8 KV-cache score rows/s (decode, 8 seq x 32768 x 512, 61 layers)",
              "qsa": "Qwen QSA KV-cache decode update_and_fetch, context rows/s (8 seq x 32768, 12 layers)",
              "linear": "dense MXFP8 linear rows/s (K 5120 -> N 5120, decode rows T = 1, 4, 16)"}.get(
                  args.workload, f"MoE layer tok/s ({args.workload})")

    if args.impl == "reference":
        if rank != 0:
            return
        r = cpu_reference(args, steps=args.steps, warmup=args.warmup, budget_s=REF_BUDGET_S)
        line = {"impl": "reference", "metric": metric, "value": round(r["value"], 3), "unit": unit,
                "n_gpus": args.gpus, "steps": r["steps"], "warmup": r["warmup"],
                "ms_per_step": round(r["sec_per_step"] * 1e3, 3), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": workload_dtype(args.workload), "data": workload_data(args.workload),
                "config": workload_config(args, args.gpus),
                "cpu_baseline": {"value": round(r["value"], 3), "unit": unit, "cores": r["cores"], "kind": "port",
                                 "sample": r["sample"]},
                "e2e": {"value": round(r["value"], 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "note": ("reference MLX CPU backend unavailable (mlx not installable offline); the oracle's "
                         "restatement timed on the host cores; steps and warmup are the counts actually run")}
        print(json.dumps(line), flush=True)
        return

    import torch
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local)
    r = run_ep(args, rank, world, dev) if _ep(args, world) else run_ours(args, rank, world, dev)
    ms = r["ms"]
    if world > 1:
        t = torch.tensor([ms, r["ms_e2e"] or 0.0, r["ms_exp"]], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, ms_e2e, ms_exp = t.tolist()
    else:
        ms_e2e, ms_exp = r["ms_e2e"], r["ms_exp"]
    value = r["tokens"] * world / (ms * 1e-3)
    if rank == 0:
        hbm = r["hbm"]
        achieved = r["alg_bytes"] / (ms_exp * 1e-3) / 1e9
        # DRAM bytes per step of the dominant kernel: per-expert traffic measured by
        # ncu on a smaller case (profiles/traffic.json), scaled by the distinct
        # experts this workload streams per step
        traffic = None
        prof = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(prof) and (r.get("distinct") or args.workload in ("qsa", "linear", "kv", "kv_scores")):
            try:
                t = json.load(open(prof)).get(args.workload)
                if t and r.get("distinct"):
                    traffic = round(t["bytes_per_expert"] * sum(r["distinct"]))
                elif t and "bytes_per_call" in t:
                    # DRAM bytes of one call of the dominant kernel, captured at the bench's own size
                    traffic = round(t["bytes_per_call"] * t.get("calls_per_step", 1))
                elif t:
                    # DRAM bytes per algorithmic byte, from one capture at a smaller size
                    traffic = round(t["dram_per_algorithmic_byte"] * r["alg_bytes"])
            except Exception:
                traffic = None
        if r.get("prefill"):
            # prefill is compute-bound: useful FLOPs of the expert FFN over the measured
            # dense bf16 tensor peak (the block-scaled MMAs run two e4m3 terms of the
            # tokens, twice these FLOPs in 8-bit tensor work at twice the 16-bit rate)
            achieved_tf = r["flops"] / (ms_exp * 1e-3) / 1e12
            roof = {"bound": "tensor", "achieved": round(achieved_tf, 1), "peak": r["tc"], "unit": "TFLOP/s",
                    "frac": round(achieved_tf / r["tc"], 4), "traffic": traffic,
                    "algorithmic_flops_per_step": r["flops"],
                    "kernel": r["kernel"] + ", " + r["peak_src"] + " dense bf16 peak (the rate of the two-term "
                              "e4m3 token operand)"}
        elif r.get("ep") and not r.get("decode"):
            roof = None
        else:
            roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                    "frac": round(achieved / hbm, 4), "traffic": traffic,
                    "algorithmic_bytes_per_step": round(r["alg_bytes"]),
                    "kernel": r["kernel"] + ", " + r["peak_src"] + " HBM peak"}
        line = {
            "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": workload_dtype(args.workload), "data": workload_data(args.workload),
            "config": workload_config(args, world),
            "e2e": None if ms_e2e is None else {"value": round(r["tokens"] * world / (ms_e2e * 1e-3), 2),
                                                 "unit": unit, "h2d_bytes_per_step": r["h2d"],
                                                 "d2h_bytes_per_step": r["d2h"]},
            "roofline": roof,
            "gpu_launches": r["launches"] * args.steps,
            "clocks": r["clocks"],
            "breakdown": r.get("breakdown", {}),
        }
        if not args.no_cpu_baseline and world == 1:
            try:
                cb = cpu_reference(args, steps=3, warmup=1, budget_s=BASELINE_BUDGET_S)
                line["cpu_baseline"] = {"value": round(cb["value"], 3), "unit": unit, "cores": cb["cores"],
                                        "kind": "port", "sample": cb["sample"]}
            except Exception as exc:  # pragma: no cover
                line["cpu_baseline"] = {"error": str(exc)}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
