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

Remote rows always land in local HBM through the collective before a kernel
reads them: no kernel touches another GPU's memory.  The local expert compute
is a callable so the same exchange logic runs on CPU ranks (gloo) in tests.
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


def plan_dispatch(idx: torch.Tensor, n_routed: int, world: int, group=None) -> EPPlan:
    """Destination ranks of each (token, slot), stable order and split sizes."""
    per = n_routed // world
    flat = idx.reshape(-1).to(torch.int64)
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

    def __init__(self, router, local_experts, n_routed: int, shared=None, group=None):
        self.router = router
        self.local_experts = local_experts
        self.n_routed = n_routed
        self.shared = shared
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.e0, self.per = shard_bounds(n_routed, self.world, self.rank)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        w, idx = self.router(x)
        k = idx.shape[-1]
        plan = plan_dispatch(idx, self.n_routed, self.world, self.group)
        src_tok = plan.order // k
        rows = x.index_select(0, src_tok)
        ids = (idx.reshape(-1).to(torch.int64).index_select(0, plan.order) % self.per).to(torch.int32)
        recv_rows = exchange(rows, plan.send_counts, plan.recv_counts, self.group)
        recv_ids = exchange(ids, plan.send_counts, plan.recv_counts, self.group)
        y = self.local_experts(recv_rows, recv_ids) if recv_rows.shape[0] else recv_rows.new_empty((0, H))
        back = exchange(y, plan.recv_counts, plan.send_counts, self.group)
        # back[i] is the output of assignment plan.order[i]
        per_assign = torch.empty((T * k, H), dtype=torch.float32, device=x.device)
        per_assign.index_copy_(0, plan.order, back.float())
        out = (per_assign.view(T, k, H) * w.reshape(T, k, 1).float()).sum(1)
        if self.shared is not None:
            out = out + self.shared(x).float()
        return out.to(torch.bfloat16)


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


def shard_experts(batched, rank: int, world: int, n_routed: int, has_shared: bool = True):
    """Slice a full BatchedExperts / QwenBatchedExperts into this rank's routed
    experts plus the shared expert (kept as the last local expert)."""
    from . import experts as X
    e0, per = shard_bounds(n_routed, world, rank)
    sel = list(range(e0, e0 + per)) + ([n_routed] if has_shared else [])
    ix = torch.tensor(sel, device=(batched.gate_up if isinstance(batched, X.QwenBatchedExperts) else batched.w2).device)
    if isinstance(batched, X.QwenBatchedExperts):
        return X.QwenBatchedExperts(*(t.index_select(0, ix).contiguous()
                                      for t in (batched.gate_up, batched.gate_up_scales, batched.down, batched.down_scales)))
    w13, s13, _ = batched.fused()
    return X.BatchedExperts(None, None, batched.w2.index_select(0, ix).contiguous(),
                            batched.w2_scales.index_select(0, ix).contiguous(), None, None,
                            w13.index_select(0, ix).contiguous(), s13.index_select(0, ix).contiguous())
