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
         gather, tcgen05 up-projection + SwiGLU, tcgen05 down-projection,
         combine; the two tcgen05 launches carry ~90% of its device time):
         algorithmic bytes (distinct experts x 23,396,352 B + activations) /
         its CUDA-event time, against the measured HBM copy bandwidth
Decode batches are replayed as CUDA graphs (one per layer and batch size),
prefill runs eagerly.
  cpu_baseline  the oracle's C restatement (OpenMP, all host threads) on a
         bounded sample of the same sweep

Other workloads: --workload ds_prefill (4096 tokens), qn_decode (B 1 and 32),
qn_prefill (16384 tokens), tiny (64 tokens, affine-4), kv (FP8 KV quantize +
dequantize of 32768 x 8 x 61 rows of 576), kv_scores (MXFP8 cache scores),
qsa (Qwen QSA affine KV caches: one decode update_and_fetch of 8 sequences at
a 32768-token context over the 12 full-attention layers), linear (dense MXFP8
linear, K = N = 5120: decode rows 1, 4, 16; 4096 in the breakdown).

`--impl reference` times the reference's algorithm on the host cores (the
oracle port; the MLX CPU backend the reference would use is not installable
here) on the same workload and prints the same JSON line with "impl".

Multi-GPU (torchrun): the MoE workloads run expert-parallel (`whallm_b200.ep`):
each rank routes its own tokens (weak scaling); the routed experts are dealt to
the ranks by popularity, equal counts per rank (WM_EP_PLACEMENT=contiguous for
plain ranges); decode gathers every rank's tokens and returns partial sums over
peer memory (WM_EP_EXCHANGE=nccl for NCCL collectives), prefill moves token rows
to the owning rank and back through NCCL all-to-all; the shared expert is
replicated; value = all ranks' tokens / max rank time.  Other workloads run as
independent replicas.
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
SWEEP = (1, 4, 16, 64)


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


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


def run_ours(args, rank, world, dev):
    import torch
    import whallm_b200 as W
    from whallm_b200 import experts as X
    from whallm_b200 import synthetic as S
    from whallm_b200.graphs import CapturedLayer

    torch.cuda.set_device(dev)
    hbm, tc, peak_src = _peaks()
    wl = args.workload
    n_layers = args.layers
    res = {}
    if wl in ("ds_decode", "ds_prefill", "qn_decode", "qn_prefill", "tiny"):
        name = {"ds_decode": "ds", "ds_prefill": "ds", "qn_decode": "qn", "qn_prefill": "qn", "tiny": "tiny"}[wl]
        if name == "tiny":
            n_layers = max(n_layers, 12)     # 14.2 MB of experts per layer: 12 layers exceed L2
        layers = [S.make_layer(name, dev, seed=1000 * rank + 17 * i, E=args.experts) for i in range(n_layers)]
        cfg = layers[0].cfg
        H = cfg["H"]
        batches = {"ds_decode": SWEEP, "ds_prefill": (4096,), "qn_decode": (1, 32), "qn_prefill": (16384,),
                   "tiny": (64,)}[wl]
        xs = [S.make_tokens(B, H, 100 + rank, dev) for B in batches]
        expert_bytes = {"ds": DS_EXPERT_BYTES, "qn": QN_EXPERT_BYTES, "tiny": 884736}[name]
        # distinct experts each (layer, batch) reads, for the algorithmic byte count
        distinct = [0.0] * len(xs)
        routes = []
        for li, lay in enumerate(layers):
            row = []
            for b, x in enumerate(xs):
                if name == "ds":
                    w, idx = lay.layer.gate(x)
                    sw = None
                else:
                    w, idx, sw = W.qwen_route(x, lay.gate_weight, cfg["k"], True, shared_gate=lay.shared_gate,
                                              logit_bias=lay.logit_bias)
                row.append((w, idx, sw))
                distinct[b] += (len(set(idx.flatten().tolist())) + (1 if cfg["shared"] else 0)) / n_layers
            routes.append(row)
        tokens_per_step = sum(batches)
        act_bytes = [x.numel() * 2 * 2 for x in xs]          # x in + out (bf16)
        alg_bytes = [d * expert_bytes + a for d, a in zip(distinct, act_bytes)]

        limit = 10.0 if name == "ds" else 0.0
        shared_id = cfg["E"] if cfg["shared"] else -1

        def experts_call(li, b, x):
            w, idx, sw = routes[li][b]
            return X.experts_forward(x, idx, layers[li].experts, weights=w, shared_expert=shared_id, shared_w=sw,
                                     swiglu_limit=limit)

        graphed = wl in ("ds_decode", "qn_decode", "tiny")
        if graphed:
            # decode (and the 64-token tiny layer): one CUDA graph per (layer, batch)
            # for the whole layer and for the expert call alone (launch overhead
            # exceeds the work)
            caps = [[CapturedLayer(lay.layer, x) for x in xs] for lay in layers]
            ecaps = [[CapturedLayer(lambda xx, li=li, b=b: experts_call(li, b, xx), x) for b, x in enumerate(xs)]
                     for li in range(n_layers)]

            def step(i):
                for c in caps[i % n_layers]:
                    c()

            def experts_only(i):
                for c in ecaps[i % n_layers]:
                    c()

            def one(i, b):
                caps[i % n_layers][b]()
        else:
            def step(i):
                lay = layers[i % n_layers]
                for x in xs:
                    lay.layer(x)

            def experts_only(i):
                for b, x in enumerate(xs):
                    experts_call(i % n_layers, b, x)

            def one(i, b):
                layers[i % n_layers].layer(xs[b])

        for i in range(args.warmup):
            step(i)
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
            step(i)
        e.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.steps
        # expert-call roofline: time the expert calls alone, same stream
        torch.cuda.synchronize()
        s2, e2 = _events(torch)
        s2.record()
        for i in range(args.steps):
            experts_only(i)
        e2.record()
        torch.cuda.synchronize()
        ms_exp = s2.elapsed_time(e2) / args.steps
        clocks = clk.stop() if clk else None
        # per-batch breakdown: back-to-back calls of one batch size (cycling the
        # layers, as in the timed step), the whole layer and the expert call alone;
        # hbm_frac is the expert call's algorithmic bytes over its time
        def one_expert(i, b):
            if graphed:
                ecaps[i % n_layers][b]()
            else:
                experts_call(i % n_layers, b, xs[b])

        per_b = {}
        reps = max(2 * n_layers, min(args.steps, 64))
        for b, x in enumerate(xs):
            tb = {}
            for name_, fn in (("layer", one), ("experts", one_expert)):
                torch.cuda.synchronize()
                s3, e3 = _events(torch)
                s3.record()
                for i in range(reps):
                    fn(i, b)
                e3.record()
                torch.cuda.synchronize()
                tb[name_] = s3.elapsed_time(e3) / reps
            per_b[str(batches[b])] = {"ms": round(tb["layer"], 4), "tok_s": round(batches[b] / tb["layer"] * 1e3, 1),
                                      "expert_ms": round(tb["experts"], 4),
                                      "distinct_experts": round(distinct[b], 2),
                                      "hbm_frac": round(alg_bytes[b] / (tb["experts"] * 1e-3) / (hbm * 1e9), 4)}
        # e2e through the public API with host buffers
        hx = [x.cpu().pin_memory() for x in xs]
        houts = [torch.empty(x.shape, dtype=torch.bfloat16).pin_memory() for x in xs]
        torch.cuda.synchronize()
        if graphed:
            ms_e2e = _e2e_overlapped(torch, dev, caps, hx, houts, args.steps)
        else:
            s4, e4 = _events(torch)
            s4.record()
            for i in range(args.steps):
                lay = layers[i % n_layers]
                for b in range(len(xs)):
                    houts[b].copy_(lay.layer(hx[b].to(dev, non_blocking=True)), non_blocking=True)
            e4.record()
            torch.cuda.synchronize()
            ms_e2e = s4.elapsed_time(e4) / args.steps
        h2d = sum(x.numel() * 2 for x in xs)
        flops = sum(B * (cfg["k"] + (1 if cfg["shared"] else 0)) * 6 * cfg["H"] * cfg["I"] for B in batches)
        res.update(dict(ms=ms, ms_exp=ms_exp, ms_e2e=ms_e2e, tokens=tokens_per_step, alg_bytes=sum(alg_bytes),
                        flops=flops, tc_peak=tc, prefill=wl in ("ds_prefill", "qn_prefill"),
                        per_b=per_b, clocks=clocks, h2d=h2d, d2h=h2d, cfg=cfg, batches=batches,
                        distinct=distinct, hbm=hbm, peak_src=peak_src,
                        launches=len(xs) * (2 + 5) if name != "tiny" else len(xs) * (2 + 4),
                        graphed=graphed, n_layers=n_layers,
                        layer_bytes=(cfg["E"] + (1 if cfg["shared"] else 0)) * expert_bytes))
        return res
    if wl == "kv_scores":
        # decode scores of one query per sequence against an MXFP8 latent cache:
        # 8 sequences x 32768 cached tokens x 512 dims per layer, 61 layers (each its own cache)
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
        s, e = _events(torch)
        s.record()
        for _ in range(args.steps):
            for li in range(n_layer):
                W.kv_scores(q, *caches[li], "mxfp8", out=out)
        e.record()
        torch.cuda.synchronize()
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
                        per_b={}, clocks=None, flops=0, h2d=Bq * D * 2 * n_layer, d2h=Bq * Lc * 2 * n_layer,
                        cfg={"B": Bq, "L": Lc, "D": D, "layers": n_layer}, batches=(), distinct=[], hbm=hbm,
                        peak_src=peak_src, launches=3 * n_layer))
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
        res.update(dict(ms=ms, ms_exp=ms_exp, ms_e2e=ms_e2e, tokens=Bq * Lc * n_layer, alg_bytes=alg, per_b={},
                        clocks=clocks, flops=0, h2d=h2d, d2h=d2h,
                        cfg={"B": Bq, "L": Lc, "layers": n_layer, "caches": [list(x) for x in shapes]}, batches=(),
                        distinct=[], hbm=hbm, peak_src=peak_src, launches=4 * n_layer,
                        kernel="history fetch of every QSA cache (k_affine_kv_fetch, K and V in one launch)",
                        dtype="u32 packed affine 8/4-bit, bf16 scales/biases, bf16 out",
                        data="synthetic (seeded N(0,1) bf16 keys/values)",
                        config={"sequences": Bq, "context": Lc, "full_attention_layers": n_layer,
                                "caches": "K/V 8-bit 2 heads x 256, index 4-bit 1 head x 128, group 32",
                                "step": "append one row per sequence + fetch the whole history, every cache",
                                "l2": f"{rd / 1e9:.1f} GB of packed history read and {wr / 1e9:.1f} GB of bf16 "
                                      "written per step: larger than L2",
                                "launch": "eager"}))
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
        # decode calls are a few microseconds of GPU work each: one CUDA graph per
        # (rows, matrix), as a decode step would replay them
        graphs = {}
        for j in range(len(sweep)):
            for li, m in enumerate(mats):
                fn = (lambda x, m=m, o=outs[j]: W.mx_linear(x, m.weight, m.scales, "mxfp8", out=o))
                graphs[j, li] = CapturedLayer(fn, xs_l[j])

        def lstep(i):
            for j in range(len(sweep)):
                graphs[j, (3 * i + j) % 8]()

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
            torch.cuda.synchronize()
            s3, e3 = _events(torch)
            s3.record()
            for i in range(32):
                graphs[j, i % 8]()
            e3.record()
            torch.cuda.synchronize()
            t_ms = s3.elapsed_time(e3) / 32
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
                ho[j].copy_(graphs[j, (3 * i + j) % 8](hx[j]), non_blocking=True)
        e4.record()
        torch.cuda.synchronize()
        ms_e2e = s4.elapsed_time(e4) / args.steps
        res.update(dict(ms=ms, ms_exp=ms, ms_e2e=ms_e2e, tokens=sum(sweep), alg_bytes=alg, per_b=per_b,
                        clocks=clocks, flops=0, h2d=sum(T * K * 2 for T in sweep), d2h=sum(T * N * 2 for T in sweep),
                        cfg={}, batches=sweep, distinct=[], hbm=hbm, peak_src=peak_src, launches=3 * len(sweep),
                        kernel="dense MXFP8 linear call (wmx_linear: token split, tcgen05 block-scaled GEMM split "
                               "over K, ordered sum of the K splits)",
                        dtype="e4m3 weights with E8M0 per 32, bf16 activations, fp32 accumulate",
                        data="synthetic (seeded N(0,0.02) weights quantized to MXFP8, N(0,1) bf16 rows)",
                        config={"K": K, "N": N, "rows_per_step": list(sweep), "weight_matrices_cycled": 8,
                                "l2": "8 x 27 MB of weights cycled: larger than L2",
                                "launch": "CUDA graph per (rows, matrix); the 4096-row calls eager",
                                "per_batch": per_b}))
        return res
    if wl == "kv":
        D, rows_total = 576, 32768 * 8 * 61
        chunk = 32768 * 8          # one layer of the 8 x 32768-token context per call
        x = torch.randn(chunk, D, device=dev).to(torch.bfloat16)
        p, sc = W.kv_quantize(x, "fp8_f32_b64")
        out = torch.empty_like(x)
        for _ in range(args.warmup):
            W.kv_quantize(x, "fp8_f32_b64", p, sc)
            W.kv_dequantize(p, sc, "fp8_f32_b64", out)
        torch.cuda.synchronize()
        s, e = _events(torch)
        s.record()
        for _ in range(args.steps):
            for _l in range(61):
                W.kv_quantize(x, "fp8_f32_b64", p, sc)
                W.kv_dequantize(p, sc, "fp8_f32_b64", out)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.steps
        per_entry = 576 + 9 * 4 + 1152
        alg = rows_total * per_entry * 2  # quantize (read bf16, write packed) + dequant (read packed, write bf16)
        res.update(dict(ms=ms, ms_exp=ms, ms_e2e=None, tokens=rows_total, alg_bytes=alg, per_b={}, clocks=None, flops=0,
                        h2d=0, d2h=0, cfg={"D": D}, batches=(), distinct=[], hbm=hbm, peak_src=peak_src,
                        launches=2 * 61))
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
    name = {"ds_decode": "ds", "ds_prefill": "ds", "qn_decode": "qn", "qn_prefill": "qn"}[wl]
    batches = {"ds_decode": SWEEP, "ds_prefill": (4096,), "qn_decode": (1, 32), "qn_prefill": (16384,)}[wl]
    decode = wl in ("ds_decode", "qn_decode")
    # decode exchanges over peer memory (CUDA IPC + flags) unless WM_EP_EXCHANGE=nccl
    peer = decode and os.environ.get("WM_EP_EXCHANGE", "peer") != "nccl"
    n_layers = args.layers
    # experts dealt to the ranks by popularity (the router's per-expert bias),
    # unless WM_EP_PLACEMENT=contiguous
    balanced = os.environ.get("WM_EP_PLACEMENT", "balanced") != "contiguous"
    moes = []
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
        if not peer:
            moes[-1].route_fn = router
        del lay
        torch.cuda.empty_cache()
    H = cfg["H"]
    E = cfg["E"]
    e0, per = EP.shard_bounds(E, world, rank)
    xs = [S.make_tokens(B, H, 100 + rank, dev) for B in batches]
    # algorithmic bytes: the distinct local experts each (layer, batch) touches
    # over all ranks' tokens, plus the shared expert, plus activations
    expert_bytes = DS_EXPERT_BYTES if name == "ds" else QN_EXPERT_BYTES
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
    if bufs is not None:
        bufs.check()
        del moes
        bufs.close()
    h2d = sum(x.numel() * 2 for x in xs)
    return dict(ms=ms, ms_exp=ms, ms_e2e=ms_e2e, tokens=sum(batches), alg_bytes=alg_bytes, per_b={}, clocks=clocks,
                h2d=h2d, d2h=h2d, cfg=cfg, batches=batches, distinct=distinct, hbm=hbm, peak_src=peak_src,
                launches=len(xs) * ((11 if peer else 7) if decode else 9), flops=0, ep=True, decode=decode,
                placement="popularity-balanced (snake order by router bias)" if balanced else "contiguous",
                launch=("CUDA graph per (layer, batch): peer-memory exchange (CUDA IPC, flags), partial experts"
                        if peer else "CUDA graph per (layer, batch): NCCL all-gather, partial experts, "
                        "reduce-scatter") if decode else "eager (NCCL all-to-all)")


# --------------------------------------------------------------------------
# reference arm: the oracle port on the host cores
# --------------------------------------------------------------------------

def cpu_reference(args, sample_steps=None):
    """Times the oracle's restatement of the reference MoE layer (router, grouped
    expert matmuls that dequantize in the loop, weighted combine, shared expert)
    on the host cores, on the same synthetic layer the device arm uses (layer 0
    of rank 0: built with the library's generator on the GPU when one is present,
    then copied to host memory before timing)."""
    import numpy as np
    import torch
    from oracle import formats as F
    from oracle import moe as M
    from oracle import router as R
    from whallm_b200 import synthetic as S

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
        name = {"ds_decode": "ds", "ds_prefill": "ds", "qn_decode": "qn", "qn_prefill": "qn", "tiny": "tiny"}[wl]
        batches = {"ds_decode": SWEEP, "ds_prefill": (256,), "qn_decode": (1, 32), "qn_prefill": (1024,),
                   "tiny": (64,)}[wl]
        dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
        if dev.type != "cuda":
            raise RuntimeError("the CPU arm builds its synthetic layer with the device generator")
        lay = S.make_layer(name, dev, seed=0)
        cfg = lay.cfg
        H, E, k = cfg["H"], cfg["E"], cfg["k"]
        xs_t = [S.make_tokens(B, H, 100, dev) for B in batches]
        xs = [x.float().cpu().numpy() for x in xs_t]
        bits = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)
        wg = bits(lay.gate_weight)
        lb = None if lay.logit_bias is None else lay.logit_bias.cpu().numpy()
        sg = None if lay.shared_gate is None else bits(lay.shared_gate).reshape(-1)
        if name == "tiny":
            a = lay.experts
            ex = M.Affine4Experts(a.w13.cpu().numpy().view(np.uint32), bits(a.w13_scales), bits(a.w13_biases),
                                  a.w2.cpu().numpy().view(np.uint32), bits(a.w2_scales), bits(a.w2_biases),
                                  M.GATE_UP, 0.0, 64)
        else:
            g = lay.experts
            w13 = g.w13 if name == "ds" else g.gate_up
            s13 = g.w13_scales if name == "ds" else g.gate_up_scales
            w2 = g.w2 if name == "ds" else g.down
            s2 = g.w2_scales if name == "ds" else g.down_scales
            ex = M.MXFP4Experts(w13.cpu().numpy(), s13.cpu().numpy(), w2.cpu().numpy(), s2.cpu().numpy(),
                                M.UP_GATE if name == "ds" else M.GATE_UP, 10.0 if name == "ds" else 0.0)
        del lay
        torch.cuda.empty_cache()

        def step():
            for x in xs:
                xb = F.f32_to_bf16_bits(x)
                if name == "ds":
                    _, idx, w, _ = R.route(xb, wg, k, R.SCORE_SQRTSOFTPLUS, logit_bias=lb, norm_eps=1e-20,
                                           route_scale=1.5)
                    M.moe_forward(x, idx, w, ex, shared_expert=E)
                elif name == "qn":
                    _, idx, w, sh = R.route(xb, wg, k, R.SCORE_SOFTMAX_BF16, logit_bias=lb, norm_eps=0.0,
                                            wg_shared_bits=sg)
                    M.moe_forward(x, idx, w, ex, shared_expert=E, shared_weight=sh)
                else:
                    _, idx, w, _ = R.route(xb, wg, k, R.SCORE_SOFTMAX_BF16, norm_eps=0.0)
                    M.moe_forward(x, idx, w, ex)

        tokens = sum(batches)
        sample = (f"{wl}: batches {list(batches)} ({tokens} tokens) on the full-size layer; oracle router + "
                  f"C expert matmuls with in-loop dequant, {threads} threads")
    step()
    steps = sample_steps or max(1, args.steps)
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    # the KV restatements are single-threaded numpy; the MoE arm runs the C kernels on every host thread
    cores = 1 if wl in ("kv", "kv_scores", "qsa", "linear") else threads
    return dict(value=tokens / dt, sec_per_step=dt, tokens=tokens, cores=cores, sample=sample)


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
        r = cpu_reference(args, sample_steps=max(1, min(args.steps, 3)))
        line = {"impl": "reference", "metric": metric, "value": round(r["value"], 3), "unit": unit, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["sec_per_step"] * 1e3, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic", "config": {"workload": args.workload},
                "cpu_baseline": {"value": round(r["value"], 3), "unit": unit, "cores": r["cores"], "kind": "port",
                                 "sample": r["sample"]},
                "e2e": {"value": round(r["value"], 3), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "note": "reference MLX CPU backend unavailable (mlx not installable offline); oracle port timed"}
        print(json.dumps(line), flush=True)
        return

    import torch
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local)
    use_ep = world > 1 and args.workload in ("ds_decode", "ds_prefill", "qn_decode", "qn_prefill")
    r = run_ep(args, rank, world, dev) if use_ep else run_ours(args, rank, world, dev)
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
        if r.get("prefill"):
            # prefill is compute-bound: useful FLOPs of the expert FFN over the measured
            # dense bf16 tensor peak (the block-scaled MMAs run two e4m3 terms of the
            # tokens, twice these FLOPs in tensor work)
            achieved_tf = r["flops"] / (ms_exp * 1e-3) / 1e12
        # DRAM bytes per step of the expert calls: per-expert traffic measured by
        # ncu on a smaller case (profiles/traffic.json), scaled by the distinct
        # experts this workload streams per step
        traffic = None
        prof = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(prof) and (r.get("distinct") or args.workload in ("qsa", "linear")):
            try:
                t = json.load(open(prof)).get(args.workload)
                if t and r.get("distinct"):
                    traffic = round(t["bytes_per_expert"] * sum(r["distinct"]))
                elif t and "bytes_per_call" in t:
                    # DRAM bytes of one call of the dominant kernel, captured at the bench's own size
                    traffic = round(t["bytes_per_call"] * t.get("calls_per_step", 1))
                elif t:
                    # DRAM bytes per algorithmic byte of the fetch, from one capture at a smaller context
                    traffic = round(t["dram_per_algorithmic_byte"] * r["alg_bytes"])
            except Exception:
                traffic = None
        if r.get("ep"):
            line_ep = {
                "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "mxfp4 weights, bf16 activations, fp32 accumulate",
                "data": "synthetic (seeded N(0,0.02) MXFP4 experts, N(0,1) bf16 tokens, Zipf-skewed router)",
                "config": {"workload": args.workload, "batches": list(r["batches"]), "tokens_per_rank": r["tokens"],
                           "layers_cycled": args.layers, "parallelism": f"ep{world}",
                           "experts_per_rank": r["cfg"]["E"] // world,
                           "placement": r.get("placement", "contiguous"),
                           "launch": r.get("launch", "eager (NCCL all-to-all)")},
                "e2e": {"value": round(r["tokens"] * world / (ms_e2e * 1e-3), 2), "unit": unit,
                        "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
                "roofline": ({"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                              "frac": round(achieved / hbm, 4), "traffic": traffic,
                              "algorithmic_bytes_per_step": round(r["alg_bytes"]),
                              "kernel": "whole layer per rank (router, collectives, expert share), "
                                        + r["peak_src"] + " HBM peak"} if r.get("decode") else None),
                "gpu_launches": r["launches"] * args.steps, "clocks": r["clocks"],
            }
            print(json.dumps(line_ep), flush=True)
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
            return
        config = {"workload": args.workload, "batches": list(r["batches"]),
                  "tokens_per_step": r["tokens"], "layers_cycled": r.get("n_layers", args.layers),
                  "l2": (f"{r.get('n_layers', args.layers)} resident layers "
                         f"({r.get('n_layers', args.layers) * r.get('layer_bytes', 0) / 1e9:.2f} GB of experts) "
                         "cycled per step: weights larger than L2"),
                  "parallelism": "replicas" if world > 1 else "single GPU",
                  "launch": "CUDA graph per (layer, batch)" if r.get("graphed") else "eager",
                  "per_batch": r["per_b"]}
        if r.get("config"):
            config = dict(r["config"], workload=args.workload,
                          parallelism="replicas" if world > 1 else "single GPU")
        line = {
            "metric": metric, "value": round(value, 2), "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": r.get("dtype", "mxfp4 weights, bf16 activations, fp32 accumulate"),
            "data": r.get("data", "synthetic (seeded N(0,0.02) MXFP4 experts, N(0,1) bf16 tokens, Zipf-skewed router)"),
            "config": config,
            "e2e": None if ms_e2e is None else {"value": round(r["tokens"] * world / (ms_e2e * 1e-3), 2),
                                                 "unit": unit, "h2d_bytes_per_step": r["h2d"],
                                                 "d2h_bytes_per_step": r["d2h"]},
            "roofline": ({"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                          "frac": round(achieved / hbm, 4), "traffic": traffic,
                          "algorithmic_bytes_per_step": r["alg_bytes"],
                          "kernel": r.get("kernel", "expert FFN call (wmoe_mxfp4_moe_forward)") + ", " +
                                    r["peak_src"] + " HBM peak"}
                         if not r.get("prefill") else
                         {"bound": "tensor", "achieved": round(achieved_tf, 1), "peak": r["tc_peak"],
                          "unit": "TFLOP/s", "frac": round(achieved_tf / r["tc_peak"], 4), "traffic": traffic,
                          "algorithmic_flops_per_step": r["flops"],
                          "kernel": "expert FFN call (wmoe_mxfp4_moe_forward), " + r["peak_src"] +
                                    " dense bf16 peak (f16 MMA)"}),
            "gpu_launches": r["launches"] * args.steps,
            "clocks": r["clocks"],
        }
        if not args.no_cpu_baseline and world == 1:
            try:
                cb = cpu_reference(args, sample_steps=1)
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
