"""Expert parallelism vs the single-GPU layer.

* One GPU, W ranks emulated: each rank's share through
  ``wmoe_mxfp4_moe_forward_ep`` (its routed experts only, the shared expert on
  its own token block, float32 partials); the sum over the ranks must match
  the full layer (``wmoe_mxfp4_moe_forward``) and the oracle, on the
  tensor-core and the CUDA-core expert paths; edge cases: a rank that owns no
  assigned expert, an id outside the layer (error path: zeros).
* Two GPUs: the all-to-all layer over NCCL (each rank routes its own tokens,
  exchanges rows, combines), the gathered decode layer over NCCL (all-gather,
  partial sums, reduce-scatter) and over peer memory (CUDA IPC rows + flags),
  eager and replayed from a CUDA graph; each
  must match the full layer on one GPU with the same weights and tokens
  (2e-2 max-relative, bf16 output).  Skipped when fewer than two GPUs are
  visible.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _partials(lay, x, world, idx=None, w=None, order=None):
    """Sum over emulated ranks of the f32 partial outputs, bf16-rounded
    (``order``: a placement order of the routed experts)."""
    from whallm_b200 import ep as EP
    from whallm_b200 import experts as X
    E = lay.cfg["E"]
    T = x.shape[0]
    if idx is None:
        w, idx = lay.layer.gate(x)
    B = T // world
    pos = EP.placement_positions(order, x.device) if order is not None else None
    acc = torch.zeros((T, x.shape[1]), dtype=torch.float32, device=x.device)
    for r in range(world):
        e0, per = EP.shard_bounds(E, world, r)
        local = EP.shard_experts(lay.experts, r, world, E, True, order=order)
        rows = (r * B, T if r == world - 1 else (r + 1) * B)
        acc += X.experts_forward(x, idx, local, weights=w, shared_expert=per, swiglu_limit=10.0,
                                 expert_range=(e0, per, E), shared_rows=rows, placement=pos)
    return acc.to(torch.bfloat16), w, idx


@pytest.mark.parametrize("world,T,H,I", [(2, 6, 1024, 256), (4, 72, 1024, 256), (8, 24, 512, 96),
                                         (2, 2, 1024, 512)])   # two tokens: the weight stream with a route filter
def test_partial_sums_over_ranks_equal_full_layer(dev, world, T, H, I):
    import sys
    sys.path.insert(0, ROOT)
    from oracle import moe as M
    from whallm_b200 import synthetic as S
    lay = S.make_layer("ds", dev, seed=11 + world, E=16, H=H, I=I)
    x = S.make_tokens(T, H, 60 + world, dev)
    got, w, idx = _partials(lay, x, world)
    full = lay.layer(x)
    assert M.max_rel_err(got.float().cpu().numpy(), full.float().cpu().numpy()) < 1e-2
    ex = M.MXFP4Experts(*(t.cpu().numpy() for t in (lay.experts.w13, lay.experts.w13_scales, lay.experts.w2,
                                                     lay.experts.w2_scales)), M.UP_GATE, 10.0)
    ref = M.moe_forward(x.float().cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), ex, shared_expert=16)
    assert M.max_rel_err(got.float().cpu().numpy(), ref) < 2e-2


@pytest.mark.parametrize("world", [2, 4, 8])
def test_partial_sums_with_balanced_placement(dev, world):
    # the same layer with experts dealt to ranks by popularity: the rank sum is unchanged
    import sys
    sys.path.insert(0, ROOT)
    from oracle import moe as M
    from whallm_b200 import ep as EP
    from whallm_b200 import synthetic as S
    lay = S.make_layer("ds", dev, seed=31 + world, E=16, H=512, I=256)
    x = S.make_tokens(24, 512, 90 + world, dev)
    order = EP.balanced_placement(lay.logit_bias.exp(), world)
    assert not torch.equal(order, torch.arange(16))               # experts really move
    got, w, idx = _partials(lay, x, world, order=order)
    plain, _, _ = _partials(lay, x, world, idx=idx, w=w)
    full = lay.layer(x)
    assert M.max_rel_err(got.float().cpu().numpy(), full.float().cpu().numpy()) < 1e-2
    assert M.max_rel_err(got.float().cpu().numpy(), plain.float().cpu().numpy()) < 1e-2


def test_partial_rank_without_assignments_and_bad_ids(dev):
    from whallm_b200 import ep as EP
    from whallm_b200 import experts as X
    from whallm_b200 import synthetic as S
    lay = S.make_layer("ds", dev, seed=4, E=8, H=512, I=256)
    x = S.make_tokens(4, 512, 9, dev)
    idx = torch.tensor([[0, 1, 2, 3, 0, 1, 2, 3]] * 4, dtype=torch.int32, device=dev)   # all on rank 0 of 2
    w = torch.full((4, 8), 0.125, device=dev)
    local1 = EP.shard_experts(lay.experts, 1, 2, 8, True)
    part = X.experts_forward(x, idx, local1, weights=w, shared_expert=4, swiglu_limit=10.0,
                             expert_range=(4, 4, 8), shared_rows=(2, 4))
    shared_only = X.experts_forward(x, torch.full((4, 1), 8, dtype=torch.int32, device=dev), lay.experts,
                                    swiglu_limit=10.0).view(4, -1).float()
    assert torch.count_nonzero(part[:2]) == 0
    assert (part[2:].to(torch.bfloat16).float() - shared_only[2:]).abs().max().item() < 1e-2 * shared_only.abs().max().item()
    bad = idx.clone()
    bad[1, 5] = 8                                           # not a routed expert of the layer
    part = X.experts_forward(x, bad, local1, weights=w, shared_expert=4, swiglu_limit=10.0,
                             expert_range=(4, 4, 8), shared_rows=(0, 4))
    assert torch.count_nonzero(part) == 0


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from oracle import moe as M
        from whallm_b200 import ep as EP
        from whallm_b200 import synthetic as S
        dev = torch.device("cuda", rank)
        lay = S.make_layer("ds", dev, seed=3, E=8, H=1024, I=256)
        x = S.make_tokens(5 + 7 * rank, 1024, 50 + rank, dev)
        full = lay.layer(x)
        local = EP.shard_experts(lay.experts, rank, world, 8, True)
        moe = EP.ExpertParallelMoE(lay.layer.gate, EP.gpu_local_experts(local, 10.0), 8,
                                   shared=EP.gpu_shared_expert(local, 8 // world, 10.0))
        got = moe(x)
        torch.cuda.synchronize()
        errs = [M.max_rel_err(got.float().cpu().numpy(), full.float().cpu().numpy())]
        # gathered decode form: same B on every rank
        from whallm_b200.graphs import CapturedLayer
        xb = S.make_tokens(9, 1024, 70 + rank, dev)
        full_b = lay.layer(xb)
        e0, per = EP.shard_bounds(8, world, rank)
        gmoe = EP.GatheredExpertParallelMoE(lay.layer.gate, EP.gpu_partial_experts(local, e0, per, 8, 10.0), 8)
        errs.append(M.max_rel_err(gmoe(xb).float().cpu().numpy(), full_b.float().cpu().numpy()))
        cap = CapturedLayer(gmoe, xb)
        y = cap(xb)
        torch.cuda.synchronize()
        errs.append(M.max_rel_err(y.float().cpu().numpy(), full_b.float().cpu().numpy()))
        del cap
        torch.cuda.synchronize()
        # the same layer with both exchanges over peer memory (CUDA IPC + flags), eager and from a graph
        bufs = EP.PeerBuffers(16, 1024, 8, device=dev)
        pmoe = EP.PeerGatheredMoE(lay.layer.gate, local, 8, 9, bufs, 10.0, True)
        errs.append(M.max_rel_err(pmoe(xb).float().cpu().numpy(), full_b.float().cpu().numpy()))
        cap = CapturedLayer(pmoe, xb)
        for _ in range(3):
            y = cap(xb)
        torch.cuda.synchronize()
        errs.append(M.max_rel_err(y.float().cpu().numpy(), full_b.float().cpu().numpy()))
        bufs.check()
        del cap
        bufs.close()
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_two_gpus_matches_single_gpu_layer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(2)])
    for p in procs:
        p.join(timeout=120)
    for rank, errs in res:
        assert len(errs) == 5 and max(errs) < 2e-2, (rank, errs)


def _ptr(t):
    import ctypes
    return ctypes.c_void_p(t.data_ptr())


def test_peer_put_wait_sum_single_rank(dev):
    """World size 1: rows land at the rank's offset, the flag is raised to the
    epoch, the wait passes and the rank-ordered sum is the rows themselves."""
    import ctypes
    import sys
    sys.path.insert(0, ROOT)
    from whallm_b200 import _lib as L
    base = ctypes.c_void_p()
    handle = (ctypes.c_ubyte * 64)()
    L.call("wep_ipc_alloc", 1 << 20, ctypes.byref(base), handle)
    try:
        buf = torch.as_tensor(_Arr(base.value, (1 << 18,), "<f4"), device=dev)      # zeroed by wep_ipc_alloc
        rows = torch.randn((5, 64), device=dev)
        ids = torch.arange(15, dtype=torch.int32, device=dev).view(5, 3)           # 12-byte rows: 4-byte copies
        flags = base.value + 4096 * 4
        ctrl = base.value + 8192 * 4
        arr = lambda ty, vals: ctypes.cast((ty * len(vals))(*vals), ctypes.c_void_p)
        st = L.stream_of(rows)
        L.call("wep_put_rows", 2, arr(ctypes.c_void_p, [rows.data_ptr(), ids.data_ptr()]),
               arr(ctypes.c_size_t, [256, 12]), None, arr(ctypes.c_size_t, [0, 2048 * 4]), 5,
               arr(ctypes.c_void_p, [base.value]), 0, 1, arr(ctypes.c_void_p, [flags]), ctypes.c_void_p(ctrl),
               ctypes.c_void_p(ctrl + 4), st)
        L.call("wep_wait", ctypes.c_void_p(flags), 1, ctypes.c_void_p(ctrl), ctypes.c_void_p(ctrl + 8), st)
        out = torch.empty((5, 64), dtype=torch.bfloat16, device=dev)
        L.call("wep_sum_rows", ctypes.c_void_p(base.value), 1, 5, 64, ctypes.c_void_p(ctrl + 8), _ptr(out), st)
        torch.cuda.synchronize()
        torch.testing.assert_close(buf[:320].view(5, 64), rows, rtol=0, atol=0)
        assert torch.equal(buf[2048:2063].view(torch.int32).view(5, 3), ids)
        ctl = buf[8192:8195].view(torch.int32).cpu().tolist()
        assert ctl == [1, 0, 0]                                                    # epoch 1, counter 0, no error
        assert int(buf[4096].view(torch.int32).item()) == 1                        # flag raised to the epoch
        torch.testing.assert_close(out, rows.to(torch.bfloat16), rtol=0, atol=0)
    finally:
        L.call("wep_ipc_free", base)


def test_peer_wait_times_out_and_reports(dev):
    """A wait on flags that nothing raises gives up after its bound (2 s), sets
    the error word and returns; the sum then writes zeros.  No fault, no hang."""
    import ctypes
    import sys
    import time
    sys.path.insert(0, ROOT)
    from whallm_b200 import _lib as L
    flags = torch.zeros(8, dtype=torch.int32, device=dev)
    epoch = torch.ones(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    part = torch.ones((2, 3, 16), dtype=torch.float32, device=dev)
    out = torch.full((3, 16), 7.0, dtype=torch.bfloat16, device=dev)
    st = L.stream_of(flags)
    torch.cuda.synchronize()
    t0 = time.time()
    L.call("wep_wait", _ptr(flags), 2, _ptr(epoch), _ptr(err), st)
    L.call("wep_sum_rows", _ptr(part), 2, 3, 16, _ptr(err), _ptr(out), st)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(err.item()) == 1
    assert 1.5 < dt < 30, dt
    assert torch.count_nonzero(out) == 0


class _Arr:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}
