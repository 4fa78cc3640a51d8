"""Expert parallelism: routed experts sharded evenly over the ranks.

The reference refuses more than one device (``_streaming_moe`` raises on a
``sharding_group``, model.py:485-486); this module is the multi-GPU form of the
same layer.  With W ranks and E routed experts, rank r owns experts
``[r*E/W, (r+1)*E/W)``; the router and the always-on shared expert are
replicated.  One forward on each rank's own tokens:

  1. route locally (bit-exact router, so every rank agrees on ids);
  2. order the (token, slot) assignments by destination rank (stable) and
     exchange per-destination counts (``all_to_all_single``, int64);
  3. send the token rows (bf16) and their local expert ids with variable
     splits (NCCL over NVLink / NVSwitch on B200s);
  4. run the local grouped expert kernel on the received rows, one assignment
     per row, un-reduced;
  5. send the expert outputs back with the reverse splits;
  6. combine on the source rank: ``sum_j w_j y_j`` in float32 plus the shared
     expert computed locally, rounded once to bf16.

In this all-to-all form remote rows land in local HBM through the collective
before a kernel reads them.  The local expert compute is a callable so the
same exchange logic runs on CPU ranks (gloo) in tests.

``GatheredExpertParallelMoE`` is the decode form: with a few tokens per rank
the all-to-all's data-dependent splits (a device-to-host read of the counts)
cost more than the rows they move, so every rank all-gathers all ranks' tokens
and routes, runs its expert share over all of them with float32 partial sums
(``wmoe_mxfp4_moe_forward_ep``: other ranks' experts skipped, the shared
expert only for its own tokens) and a reduce-scatter adds the partials back
onto the owning rank.  Every collective has a fixed size, so one decode step
of the layer is capturable as a CUDA graph.  ``PeerGatheredMoE`` does the same
exchange without a collective library: ``wep_put_rows`` stores this rank's
rows into every rank's CUDA-IPC-mapped buffer with plain stores over NVLink
and raises a flag there; ``wep_wait`` spins (bounded) on the local flags, and
``wep_sum_rows`` adds the partial sums.  Those three kernels are the only ones
that touch another GPU's memory (plain loads and stores; no TMA, no library
kernel on peer memory).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class EPPlan:
    order: torch.Tensor        # [T*k] flat assignment ids sorted by destination rank (stable)
    send_counts: list          # rows this rank sends to each rank
    recv_counts: list          # rows this rank receives from each rank


def shard_bounds(n_routed: int, world: int, rank: int):
    if n_routed % world:
        raise ValueError(f"{n_routed} experts do not shard evenly over {world} ranks")
    per = n_routed // world
    return rank * per, per


def balanced_placement(load, world: int) -> torch.Tensor:
    """Order of the routed experts for sharding: rank r owns
    ``order[r*c:(r+1)*c]`` (c = E / world).  The experts are dealt to the ranks
    hottest first in snake order (0..W-1, W-1..0, ...), so every rank holds c
    experts and about the same share of the expected load ``load`` (e.g. the
    routing popularity: exp of the router's per-expert logit bias, or counts
    from a calibration pass).  Ties go to the lower id; each rank's experts
    are kept in id order.  int64 [E] on the CPU."""
    load = torch.as_tensor(load, dtype=torch.float64).detach().cpu().reshape(-1)
    E = load.numel()
    if E % world:
        raise ValueError(f"{E} experts do not shard evenly over {world} ranks")
    hot = torch.argsort(-load, stable=True).tolist()
    ranks = [[] for _ in range(world)]
    for i, e in enumerate(hot):
        r = i % (2 * world)
        ranks[r if r < world else 2 * world - 1 - r].append(e)
    return torch.tensor([e for r in ranks for e in sorted(r)], dtype=torch.int64)


def placement_positions(order: torch.Tensor, device=None) -> torch.Tensor:
    """Inverse of a placement order: position[e] = j where order[j] = e (int32)."""
    order = torch.as_tensor(order, dtype=torch.int64).cpu()
    pos = torch.empty_like(order)
    pos[order] = torch.arange(order.numel(), dtype=torch.int64)
    if sorted(order.tolist()) != list(range(order.numel())):
        raise ValueError("placement order must be a permutation of the routed experts")
    return pos.to(torch.int32).to(device) if device is not None else pos.to(torch.int32)


def plan_dispatch(idx: torch.Tensor, n_routed: int, world: int, group=None, positions=None) -> EPPlan:
    """Destination ranks of each (token, slot), stable order and split sizes.
    ``positions`` (device int32 [n_routed], ``placement_positions``) places
    expert e at position positions[e] of the ranks' contiguous ranges."""
    per = n_routed // world
    flat = idx.reshape(-1).to(torch.int64)
    if positions is not None:
        flat = positions.to(torch.int64)[flat]
    dest = flat // per
    order = torch.sort(dest, stable=True).indices
    send = torch.bincount(dest, minlength=world).to(torch.int64)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return EPPlan(order, send.tolist(), recv.tolist())


def exchange(t: torch.Tensor, send_counts, recv_counts, group=None) -> torch.Tensor:
    """Variable-split all-to-all of rows of ``t`` ([rows, ...])."""
    out = torch.empty((sum(recv_counts),) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_to_all_single(out, t.contiguous(), output_split_sizes=list(recv_counts),
                           input_split_sizes=list(send_counts), group=group)
    return out


class ExpertParallelMoE:
    """One MoE layer with its routed experts sharded over a process group.

    ``router(x) -> (weights f32 [T, k], idx int32 [T, k])`` with global expert
    ids; ``local_experts(rows bf16 [R, H], local_ids int32 [R]) -> bf16 [R, H]``
    runs this rank's experts, one assignment per row (see ``gpu_local_experts``);
    ``shared(x) -> f32 [T, H]`` (optional) is the replicated shared expert."""

    def __init__(self, router, local_experts, n_routed: int, shared=None, group=None, positions=None,
                 reduce=None):
        self.router = router
        self.local_experts = local_experts
        # reduce(back bf16 [T*k, H], slots int32 [T, k], weights f32 [T, k], add f32 [T, H] or None) -> bf16 [T, H]:
        # the device combine by default; host-tensor ranks (gloo tests) pass their own
        self.reduce = reduce if reduce is not None else gpu_rows_reduce
        self.n_routed = n_routed
        self.shared = shared
        self.group = group
        self.positions = positions          # placement_positions(order) on the device, or None
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.e0, self.per = shard_bounds(n_routed, self.world, self.rank)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        w, idx = self.router(x)
        k = idx.shape[-1]
        add = None
        side = None
        if self.shared is not None and x.is_cuda:
            # the replicated shared expert needs no exchange: it runs on a side
            # stream while the rows travel (the router has run on the main stream)
            main = torch.cuda.current_stream(x.device)
            side = torch.cuda.Stream(device=x.device)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                add = self.shared(x).float().contiguous()
        elif self.shared is not None:
            add = self.shared(x).float().contiguous()
        plan = plan_dispatch(idx, self.n_routed, self.world, self.group, self.positions)
        src_tok = plan.order // k
        rows = x.index_select(0, src_tok)
        gid = idx.reshape(-1).to(torch.int64)
        if self.positions is not None:
            gid = self.positions.to(torch.int64)[gid]
        ids = (gid.index_select(0, plan.order) % self.per).to(torch.int32)
        recv_rows = exchange(rows, plan.send_counts, plan.recv_counts, self.group)
        recv_ids = exchange(ids, plan.send_counts, plan.recv_counts, self.group)
        y = self.local_experts(recv_rows, recv_ids) if recv_rows.shape[0] else recv_rows.new_empty((0, H))
        back = exchange(y, plan.recv_counts, plan.send_counts, self.group)
        # back[i] is the output of assignment plan.order[i]: slot of assignment (t, j) in back
        slots = torch.empty(T * k, dtype=torch.int32, device=x.device)
        slots[plan.order] = torch.arange(T * k, dtype=torch.int32, device=x.device)
        if side is not None:
            torch.cuda.current_stream(x.device).wait_stream(side)
            add.record_stream(torch.cuda.current_stream(x.device))
        return self.reduce(back.contiguous(), slots.view(T, k), w.reshape(T, k).float().contiguous(), add)


def _all_gather(t: torch.Tensor, world: int, group=None) -> torch.Tensor:
    out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    return out


def _reduce_scatter(t: torch.Tensor, world: int, rank: int, group=None) -> torch.Tensor:
    """Sum of ``t`` [world*B, ...] over the ranks, rows [rank*B, (rank+1)*B) kept."""
    B = t.shape[0] // world
    if dist.get_backend(group) == "nccl":
        out = torch.empty((B,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.reduce_scatter_tensor(out, t.contiguous(), group=group)
        return out
    s = t.clone()   # backends without reduce-scatter (gloo on CPU ranks)
    dist.all_reduce(s, group=group)
    return s[rank * B:(rank + 1) * B]


class GatheredExpertParallelMoE:
    """Decode form of the expert-parallel layer (fixed-size collectives only).

    ``router(x) -> (weights f32 [B, k], idx int32 [B, k][, shared_w f32 [B]])``
    with global expert ids; ``partial(xg, idxg, wg, swg, rows) -> f32 [W*B, H]``
    is this rank's share over all ranks' tokens (``gpu_partial_experts``),
    with the shared expert applied to rows [lo, hi) only.  Every rank must
    call with the same B."""

    def __init__(self, router, partial, n_routed: int, group=None):
        self.router = router
        self.partial = partial
        self.n_routed = n_routed
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.e0, self.per = shard_bounds(n_routed, self.world, self.rank)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        B, H = x.shape
        r = self.router(x)
        w, idx = r[0], r[1]
        sw = r[2] if len(r) > 2 else None
        k = idx.shape[-1]
        cols = [idx.reshape(B, k).to(torch.int32), w.reshape(B, k).float().contiguous().view(torch.int32)]
        if sw is not None:
            cols.append(sw.reshape(B, 1).float().contiguous().view(torch.int32))
        routes = _all_gather(torch.cat(cols, 1), self.world, self.group)
        xg = _all_gather(x, self.world, self.group)
        idxg = routes[:, :k].contiguous()
        wg = routes[:, k:2 * k].contiguous().view(torch.float32)
        swg = routes[:, 2 * k].contiguous().view(torch.float32) if sw is not None else None
        part = self.partial(xg, idxg, wg, swg, (self.rank * B, (self.rank + 1) * B))
        return _reduce_scatter(part, self.world, self.rank, self.group).to(torch.bfloat16)


class _DeviceArray:
    """A raw device pointer as a CUDA array-interface object (viewed by torch.as_tensor)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _view(ptr: int, shape, dtype):
    typestr = {torch.int16: "<i2", torch.int32: "<i4", torch.float32: "<f4", torch.uint8: "|u1"}
    if dtype == torch.bfloat16:
        return torch.as_tensor(_DeviceArray(ptr, shape, "<i2"), device="cuda").view(torch.bfloat16)
    return torch.as_tensor(_DeviceArray(ptr, shape, typestr[dtype]), device="cuda")


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class PeerBuffers:
    """One CUDA-IPC buffer per rank for the peer exchanges of the gathered
    decode layer, mapped by every rank: the gathered tokens and routes of all
    ranks (W * B_max rows), the returned partial sums ([W][B_max] rows), two
    flag arrays with their epochs and arrival counters, and an error word.
    The exchanges are lock-step, so every layer and batch size of a process
    group can share one set (calls are stream-ordered on every rank)."""

    def __init__(self, B_max: int, H: int, k: int, group=None, device=None):
        import ctypes
        from . import _lib as L
        self.L = L
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("peer exchange supports up to 8 ranks")
        self.B_max, self.H, self.k = B_max, H, k
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        W, R = self.world, self.world * B_max
        off = 0
        layout = {}
        for name, nbytes in (("x", R * H * 2), ("idx", R * k * 4), ("w", R * k * 4), ("sw", R * 4),
                             ("ret", R * H * 4), ("flags", 2 * 64 * 4), ("ctrl", 256)):
            layout[name] = off
            off = _align(off + nbytes)
        self.layout, self.nbytes = layout, off
        base = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * 64)()
        L.call("wep_ipc_alloc", off, ctypes.byref(base), handle)
        self.base = base.value
        handles = [None] * W
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.peers = []
        for q in range(W):
            if q == self.rank:
                self.peers.append(self.base)
            else:
                p = ctypes.c_void_p()
                L.call("wep_ipc_open", (ctypes.c_ubyte * 64).from_buffer_copy(handles[q]), ctypes.byref(p))
                self.peers.append(p.value)
        ctrl = self.base + layout["ctrl"]
        self.epoch = [ctrl, ctrl + 4]                  # uint32 epochs of the two exchanges
        self.counter = [ctrl + 8, ctrl + 12]           # CTA-arrival counters
        self.err_ptr = ctrl + 16
        self.err = _view(self.err_ptr, (1,), torch.int32)
        self.flags_local = [self.base + layout["flags"], self.base + layout["flags"] + 256]
        self.flags_peer = [[p + layout["flags"] + 256 * c for p in self.peers] for c in range(2)]
        dist.barrier(group=group)                      # every peer mapped before any write

    def views(self, B: int):
        """Gathered tokens / ids / weights / shared weights ([W*B] rows) and returned partials ([W, B, H])."""
        if B > self.B_max:
            raise ValueError(f"batch {B} exceeds the buffers' {self.B_max}")
        b, lay, R, H, k = self.base, self.layout, self.world * B, self.H, self.k
        return (_view(b + lay["x"], (R, H), torch.bfloat16), _view(b + lay["idx"], (R, k), torch.int32),
                _view(b + lay["w"], (R, k), torch.float32), _view(b + lay["sw"], (R,), torch.float32),
                _view(b + lay["ret"], (self.world, B, H), torch.float32))

    def put(self, ch: int, regions, rows: int, stream):
        """wep_put_rows of (src ptr, row bytes, per-peer src stride, dst offset) regions, then wep_wait."""
        import ctypes
        L = self.L
        n = len(regions)
        arr = lambda ty, vals: ctypes.cast((ty * len(vals))(*vals), ctypes.c_void_p)
        L.call("wep_put_rows", n, arr(ctypes.c_void_p, [r[0] for r in regions]),
               arr(ctypes.c_size_t, [r[1] for r in regions]), arr(ctypes.c_size_t, [r[2] for r in regions]),
               arr(ctypes.c_size_t, [r[3] for r in regions]), rows, arr(ctypes.c_void_p, self.peers), self.rank,
               self.world, arr(ctypes.c_void_p, self.flags_peer[ch]), ctypes.c_void_p(self.epoch[ch]),
               ctypes.c_void_p(self.counter[ch]), stream)
        L.call("wep_wait", ctypes.c_void_p(self.flags_local[ch]), self.world, ctypes.c_void_p(self.epoch[ch]),
               ctypes.c_void_p(self.err_ptr), stream)

    def check(self):
        """Raise if an exchange wait timed out (a rank stopped participating)."""
        if int(self.err.item()) != 0:
            raise RuntimeError("expert-parallel peer exchange timed out waiting for a rank")

    def close(self):
        """Unmap the peers' buffers and free this rank's, once every rank is done with them."""
        if getattr(self, "base", None) is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for q, p in enumerate(self.peers):
            if q != self.rank:
                self.L.call("wep_ipc_close", ctypes_ptr(p))
        dist.barrier(group=self.group)
        self.L.call("wep_ipc_free", ctypes_ptr(self.base))
        self.base = None


class PeerGatheredMoE:
    """The gathered decode layer with both exchanges over peer memory
    (``wep_put_rows`` / ``wep_wait`` / ``wep_sum_rows``) instead of
    collectives.  A call: route own B tokens -> write tokens + routes into
    every rank's buffer -> wait for all ranks' flags -> this rank's expert
    share over all W*B tokens (float32 partials) -> write each rank's block of
    partials into its buffer -> wait -> out = bf16(sum of the W partials in
    rank order).  ``router(x) -> (weights f32 [B, k], idx int32 [B, k][,
    shared_w f32 [B]])``; ``experts``: this rank's slice from
    ``shard_experts``; ``bufs``: a ``PeerBuffers`` of the group.  Every rank
    calls with the same B in the same order."""

    def __init__(self, router, experts, n_routed: int, B: int, bufs: PeerBuffers, swiglu_limit: float = 0.0,
                 has_shared: bool = True, shared_gated: bool = False, positions=None):
        self.router = router
        self.positions = positions          # placement_positions(order) on the device, or None
        self.experts = experts
        self.n_routed = n_routed
        self.B = B
        self.bufs = bufs
        self.limit = float(swiglu_limit)
        self.has_shared = has_shared
        self.shared_gated = shared_gated
        self.e0, self.per = shard_bounds(n_routed, bufs.world, bufs.rank)
        self.rx_x, self.rx_idx, self.rx_w, self.rx_sw, self.ret = bufs.views(B)
        self.part = torch.empty((bufs.world * B, bufs.H), dtype=torch.float32, device=bufs.device)
        self.out = torch.empty((B, bufs.H), dtype=torch.bfloat16, device=bufs.device)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        from . import experts as X
        bufs, L = self.bufs, self.bufs.L
        B, H, k = self.B, bufs.H, bufs.k
        if tuple(x.shape) != (B, H):
            raise ValueError(f"peer layer expects [{B}, {H}] tokens")
        r = self.router(x)
        w = r[0].reshape(B, k).float().contiguous()
        idx = r[1].reshape(B, k).to(torch.int32).contiguous()
        sw = r[2].reshape(B).float().contiguous() if (self.shared_gated and len(r) > 2) else None
        lay = bufs.layout
        xc = x.contiguous()
        regions = [(xc.data_ptr(), 2 * H, 0, lay["x"]), (idx.data_ptr(), 4 * k, 0, lay["idx"]),
                   (w.data_ptr(), 4 * k, 0, lay["w"])]
        if sw is not None:
            regions.append((sw.data_ptr(), 4, 0, lay["sw"]))
        stream = L.stream_of(self.out)
        bufs.put(0, regions, B, stream)
        X.experts_forward(self.rx_x, self.rx_idx, self.experts, weights=self.rx_w,
                          shared_expert=self.per if self.has_shared else -1,
                          shared_w=self.rx_sw if sw is not None else None, swiglu_limit=self.limit,
                          expert_range=(self.e0, self.per, self.n_routed), placement=self.positions,
                          shared_rows=(bufs.rank * B, (bufs.rank + 1) * B), out=self.part)
        bufs.put(1, [(self.part.data_ptr(), 4 * H, B * 4 * H, lay["ret"])], B, stream)
        L.call("wep_sum_rows", L.ptr(self.ret), bufs.world, B, H, ctypes_ptr(bufs.err_ptr), L.ptr(self.out), stream)
        return self.out


def ctypes_ptr(v: int):
    import ctypes
    return ctypes.c_void_p(v)


def gpu_partial_experts(experts, e0: int, per: int, n_routed: int, swiglu_limit: float = 0.0,
                        has_shared: bool = True, positions=None):
    """This rank's share on the device: ``experts`` from ``shard_experts``
    (the routed experts at placement positions [e0, e0+per) as 0..per-1, then
    the shared expert)."""
    from . import experts as X

    def run(xg, idxg, wg, swg, rows):
        return X.experts_forward(xg, idxg, experts, weights=wg, shared_expert=per if has_shared else -1,
                                 shared_w=swg, swiglu_limit=swiglu_limit, expert_range=(e0, per, n_routed),
                                 shared_rows=rows, placement=positions)
    return run


def gpu_rows_reduce(back, slots, weights, add=None):
    """The all-to-all layer's combine on the device (``wmoe_route_reduce``)."""
    from .moe import rows_reduce
    return rows_reduce(back, slots, weights, add)


def gpu_local_experts(experts, swiglu_limit: float = 0.0):
    """This rank's experts on the device: un-reduced grouped expert forward,
    one (row, expert) assignment per row (k = 1)."""
    from . import experts as X

    def run(rows: torch.Tensor, local_ids: torch.Tensor) -> torch.Tensor:
        out = X.experts_forward(rows, local_ids.view(-1, 1), experts, swiglu_limit=swiglu_limit)
        return out.view(rows.shape[0], rows.shape[1])
    return run


def gpu_shared_expert(experts, shared_index: int, swiglu_limit: float = 0.0, gate=None):
    """The replicated shared expert (stored at ``shared_index`` of ``experts``),
    scaled by ``gate(x) -> [T]`` when given (Qwen's sigmoid gate)."""
    from . import experts as X

    def run(x: torch.Tensor) -> torch.Tensor:
        T = x.shape[0]
        ids = torch.full((T, 1), shared_index, dtype=torch.int32, device=x.device)
        y = X.experts_forward(x, ids, experts, swiglu_limit=swiglu_limit).view(T, -1).float()
        return y * gate(x).view(T, 1) if gate is not None else y
    return run


def shard_experts(batched, rank: int, world: int, n_routed: int, has_shared: bool = True, order=None):
    """Slice a full BatchedExperts / QwenBatchedExperts into this rank's routed
    experts (``order[e0:e0+per]`` with a placement order, else [e0, e0+per))
    plus the shared expert (kept as the last local expert)."""
    from . import experts as X
    e0, per = shard_bounds(n_routed, world, rank)
    routed = list(range(e0, e0 + per)) if order is None else [int(e) for e in order[e0:e0 + per]]
    sel = routed + ([n_routed] if has_shared else [])
    ix = torch.tensor(sel, device=(batched.gate_up if isinstance(batched, X.QwenBatchedExperts) else batched.w2).device)
    if isinstance(batched, X.QwenBatchedExperts):
        return X.QwenBatchedExperts(*(t.index_select(0, ix).contiguous()
                                      for t in (batched.gate_up, batched.gate_up_scales, batched.down, batched.down_scales)))
    w13, s13, _ = batched.fused()
    return X.BatchedExperts(None, None, batched.w2.index_select(0, ix).contiguous(),
                            batched.w2_scales.index_select(0, ix).contiguous(), None, None,
                            w13.index_select(0, ix).contiguous(), s13.index_select(0, ix).contiguous())
