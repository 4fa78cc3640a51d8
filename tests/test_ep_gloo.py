"""Expert-parallel exchange logic on CPU ranks (gloo, world size 2).

The dispatch plan, the two variable-split all-to-alls and the combine of
``whallm_b200.ep.ExpertParallelMoE`` run for real over gloo; the router and the
local expert math are the CPU oracle, so the result must match the
single-process oracle layer on each rank's tokens.  A second test makes one
rank leave before the exchange: the other rank's collective must fail within
the process-group timeout instead of hanging (failure detection on the host,
no GPU involved).
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _host_reduce(back, slots, weights, add=None):
    """The all-to-all layer's combine for host-tensor ranks (the device kernel's
    arithmetic: float32 sum over j, then the addend)."""
    T, k = slots.shape
    rows = back.float()[slots.reshape(-1).long()].view(T, k, -1)
    out = (rows * weights.view(T, k, 1)).sum(1)
    if add is not None:
        out = out + add
    return out.to(torch.bfloat16)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _layer(seed=5, E=8, H=64, I=64, k=3):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import formats as F
    from oracle import moe as M
    rng = np.random.default_rng(seed)
    n = E + 1
    w13 = np.zeros((n, 2 * I, H // 2), np.uint8)
    s13 = np.zeros((n, 2 * I, H // 32), np.uint8)
    w2 = np.zeros((n, H, I // 2), np.uint8)
    s2 = np.zeros((n, H, I // 32), np.uint8)
    for e in range(n):
        w13[e], s13[e] = F.mxfp4_quantize_bf16(F.f32_to_bf16_bits(rng.normal(0, 0.1, (2 * I, H)).astype(np.float32)))
        w2[e], s2[e] = F.mxfp4_quantize_bf16(F.f32_to_bf16_bits(rng.normal(0, 0.1, (H, I)).astype(np.float32)))
    ex = M.MXFP4Experts(w13, s13, w2, s2, M.UP_GATE, 10.0)
    wg = F.f32_to_bf16_bits((rng.normal(0, 1, (E, H)) / np.sqrt(H)).astype(np.float32))
    return ex, wg, dict(E=E, H=H, I=I, k=k)


def _tokens(rank, T, H):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import formats as F
    rng = np.random.default_rng(100 + rank)
    return F.round_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))


def _worker(rank, world, port, result_q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import formats as F
        from oracle import moe as M
        from oracle import router as R
        from whallm_b200.ep import ExpertParallelMoE, shard_bounds
        ex, wg, c = _layer()
        E, H, k = c["E"], c["H"], c["k"]
        T = 7 + 5 * rank
        x = _tokens(rank, T, H)

        def router(xt):
            xb = F.f32_to_bf16_bits(xt.float().numpy())
            _, idx, w, _ = R.route(xb, wg, k, R.SCORE_SQRTSOFTPLUS, norm_eps=1e-20, route_scale=1.5)
            return torch.from_numpy(w), torch.from_numpy(idx)

        e0, per = shard_bounds(E, world, rank)

        def local(rows, ids):
            rows_np = rows.float().numpy()
            out = np.zeros_like(rows_np)
            for le in np.unique(ids.numpy()):
                sel = np.flatnonzero(ids.numpy() == le)
                out[sel] = ex.ffn(e0 + int(le), rows_np[sel])
            return torch.from_numpy(F.round_bf16(out)).to(torch.bfloat16)

        def shared(xt):
            return torch.from_numpy(ex.ffn(E, xt.float().numpy()))

        moe = ExpertParallelMoE(router, local, E, shared=shared, reduce=_host_reduce)
        got = moe(torch.from_numpy(x).to(torch.bfloat16)).float().numpy()
        _, idx, w, _ = R.route(F.f32_to_bf16_bits(x), wg, k, R.SCORE_SQRTSOFTPLUS, norm_eps=1e-20, route_scale=1.5)
        ref = M.moe_forward(x, idx, w, ex, shared_expert=E)
        result_q.put((rank, M.max_rel_err(got, ref), int(idx.max()), int(idx.min())))
    finally:
        dist.destroy_process_group()


def _placed_worker(rank, world, port, result_q):
    """The all-to-all layer with a popularity-balanced placement: experts move
    between ranks, the layer output must not change."""
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import formats as F
        from oracle import moe as M
        from oracle import router as R
        from whallm_b200.ep import ExpertParallelMoE, balanced_placement, placement_positions, shard_bounds
        ex, wg, c = _layer()
        E, H, k = c["E"], c["H"], c["k"]
        T = 9 + 3 * rank
        x = _tokens(rank, T, H)
        order = balanced_placement(np.arange(E, 0, -1) ** 2.0, world)   # skewed load: expert 0 hottest
        pos = placement_positions(order)

        def router(xt):
            xb = F.f32_to_bf16_bits(xt.float().numpy())
            _, idx, w, _ = R.route(xb, wg, k, R.SCORE_SQRTSOFTPLUS, norm_eps=1e-20, route_scale=1.5)
            return torch.from_numpy(w), torch.from_numpy(idx)

        e0, per = shard_bounds(E, world, rank)
        mine = [int(e) for e in order[e0:e0 + per]]

        def local(rows, ids):
            rows_np = rows.float().numpy()
            out = np.zeros_like(rows_np)
            for le in np.unique(ids.numpy()):
                sel = np.flatnonzero(ids.numpy() == le)
                out[sel] = ex.ffn(mine[int(le)], rows_np[sel])
            return torch.from_numpy(F.round_bf16(out)).to(torch.bfloat16)

        moe = ExpertParallelMoE(router, local, E, shared=lambda xt: torch.from_numpy(ex.ffn(E, xt.float().numpy())),
                                positions=pos, reduce=_host_reduce)
        got = moe(torch.from_numpy(x).to(torch.bfloat16)).float().numpy()
        _, idx, w, _ = R.route(F.f32_to_bf16_bits(x), wg, k, R.SCORE_SQRTSOFTPLUS, norm_eps=1e-20, route_scale=1.5)
        ref = M.moe_forward(x, idx, w, ex, shared_expert=E)
        result_q.put((rank, M.max_rel_err(got, ref), sorted(mine), 0))
    finally:
        dist.destroy_process_group()


def _gathered_worker(rank, world, port, result_q):
    """Decode form: all-gather tokens + routes, partial sums, reduce-scatter."""
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from oracle import formats as F
        from oracle import moe as M
        from oracle import router as R
        from whallm_b200.ep import GatheredExpertParallelMoE, shard_bounds
        ex, wg, c = _layer()
        E, H, k = c["E"], c["H"], c["k"]
        B = 6                                   # same batch on every rank
        x = _tokens(rank, B, H)
        e0, per = shard_bounds(E, world, rank)

        def router(xt):
            _, idx, w, _ = R.route(F.f32_to_bf16_bits(xt.float().numpy()), wg, k, R.SCORE_SQRTSOFTPLUS,
                                   norm_eps=1e-20, route_scale=1.5)
            sw = np.full((xt.shape[0],), 0.75, np.float32)   # a per-token shared-expert weight
            return torch.from_numpy(w), torch.from_numpy(idx), torch.from_numpy(sw)

        def partial(xg, idxg, wgt, swg, rows):
            xs = xg.float().numpy()
            ids, ws, sws = idxg.numpy(), wgt.numpy(), swg.numpy()
            out = np.zeros_like(xs)
            for t in range(xs.shape[0]):
                for j in range(k):
                    if e0 <= ids[t, j] < e0 + per:
                        out[t] += ws[t, j] * ex.ffn(int(ids[t, j]), xs[t:t + 1])[0]
                if rows[0] <= t < rows[1]:
                    out[t] += sws[t] * ex.ffn(E, xs[t:t + 1])[0]
            return torch.from_numpy(out)

        moe = GatheredExpertParallelMoE(router, partial, E)
        got = moe(torch.from_numpy(x).to(torch.bfloat16)).float().numpy()
        _, idx, w, _ = R.route(F.f32_to_bf16_bits(x), wg, k, R.SCORE_SQRTSOFTPLUS, norm_eps=1e-20, route_scale=1.5)
        ref = M.moe_forward(x, idx, w, ex, shared_expert=E, shared_weight=np.full((B,), 0.75, np.float32))
        result_q.put((rank, M.max_rel_err(got, ref), int(idx.max()), int(idx.min())))
    finally:
        dist.destroy_process_group()


def _dying_worker(rank, world, port, result_q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        # leave between steps: no collective of this rank is in flight
        result_q.put((rank, "left"))
        result_q.close()
        result_q.join_thread()  # flush the queue's feeder thread before exiting
        os._exit(0)
    from whallm_b200.ep import plan_dispatch
    try:
        plan_dispatch(torch.zeros((4, 2), dtype=torch.int32), 8, world)
        result_q.put((rank, "no error"))
    except Exception as exc:  # the survivor must see an error, not hang
        result_q.put((rank, "error: " + type(exc).__name__))


def _spawn(fn, world=2, timeout=600):
    # generous: on a freshly started machine the spawned ranks' first imports of
    # torch and the library can take minutes; a healthy run returns in seconds
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = []
    for _ in range(world):
        out.append(q.get(timeout=timeout))
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return sorted(out, key=lambda r: r[0])


def test_ep_exchange_matches_single_process_layer():
    res = _spawn(_worker)
    for rank, err, hi, lo in res:
        assert err < 2e-2, (rank, err)
        assert 0 <= lo <= hi < 8


def test_gathered_ep_matches_single_process_layer():
    res = _spawn(_gathered_worker)
    for rank, err, hi, lo in res:
        assert err < 2e-2, (rank, err)
        assert 0 <= lo <= hi < 8


def test_ep_exchange_with_balanced_placement():
    res = _spawn(_placed_worker)
    assert sorted(res[0][2] + res[1][2]) == list(range(8))      # every expert on exactly one rank
    for rank, err, _, _ in res:
        assert err < 2e-2, (rank, err)


def test_balanced_placement_properties():
    from whallm_b200.ep import balanced_placement, placement_positions
    rng = np.random.default_rng(0)
    for E, W in ((256, 8), (512, 8), (16, 4), (8, 2)):
        load = rng.zipf(1.5, E).astype(np.float64)
        order = balanced_placement(load, W)
        assert sorted(order.tolist()) == list(range(E))
        per = order.view(W, E // W)
        shares = np.array([load[r.numpy()].sum() for r in per])
        contiguous = load.reshape(W, -1).sum(1)
        assert shares.max() <= contiguous.max() + 1e-9          # never worse than contiguous ranges
        assert all(list(r) == sorted(r.tolist()) for r in per)   # each rank's experts in id order
        pos = placement_positions(order)
        assert torch.equal(order[pos.long()], torch.arange(E))
    with pytest.raises(ValueError, match="evenly"):
        balanced_placement(np.ones(10), 4)
    with pytest.raises(ValueError, match="permutation"):
        placement_positions(torch.tensor([0, 0, 1, 2]))


def test_rank_leaving_surfaces_as_collective_error():
    res = _spawn(_dying_worker)
    assert res[1][1] == "left"
    assert res[0][1].startswith("error"), res


def test_uneven_sharding_rejected():
    from whallm_b200.ep import shard_bounds
    with pytest.raises(ValueError):
        shard_bounds(10, 4, 0)
