"""Expert parallelism on 2 GPUs over NCCL vs the single-GPU layer.

Each rank holds half of the routed experts plus the shared expert, routes its
own tokens, exchanges rows with all-to-all and combines; the result must match
the full layer run on one GPU with the same weights and tokens (2e-2
max-relative, bf16 output).  Skipped when fewer than two GPUs are visible.
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
        q.put((rank, M.max_rel_err(got.float().cpu().numpy(), full.float().cpu().numpy())))
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
    for rank, err in res:
        assert err < 2e-2, (rank, err)
