"""Expert-parallel dispatch/combine across 2 and 4 CPU ranks over gloo.

The expert computation is a stand-in (each expert scales its rows by its global id
+ 1), so the test checks the exchange itself: every pair reaches the rank owning
its expert, comes back to its sender in (token, k) order, and the combine equals
the single-process answer, in both the padded (decode) and exact (prefill) modes.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, H, K = 8, 16, 2


def _fake_expert(rank, per_rank):
    def fn(rows, ids):
        g = ids.to(torch.float32) + rank * per_rank + 1.0
        return rows * torch.where(ids >= 0, g, torch.zeros_like(g))[:, None]
    return fn


def _worker(rank, world, port, T, padded, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from bigrig_b200.ep import ExpertParallel
        ep = ExpertParallel(E)
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(T, H, generator=g)
        lg = torch.randn(T, E, generator=g)
        idx = torch.topk(lg, K, dim=1).indices.to(torch.int32)
        sc = torch.softmax(torch.randn(T, K, generator=g), dim=1)
        out = ep.dispatch_combine(x, idx, sc, _fake_expert(rank, ep.per_rank), padded=padded)
        want = torch.zeros(T, H)
        for j in range(K):
            want += sc[:, j:j + 1] * x * (idx[:, j:j + 1].float() + 1.0)
        q.put((rank, float((out - want).abs().max())))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(world, T, padded):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T, padded, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=10) for _ in range(world))
    assert max(res.values()) < 1e-5, res


@pytest.mark.parametrize("padded", [True, False])
@pytest.mark.parametrize("T", [1, 5])
def test_dispatch_combine_two_ranks(padded, T):
    _run_ranks(2, T, padded)


@pytest.mark.parametrize("padded", [True, False])
def test_dispatch_combine_four_ranks(padded):
    """Two experts per rank, as bench.py's expert-parallel run places OLMoE's 64 on 4 GPUs
    in proportion: pairs cross to three peers and back."""
    _run_ranks(4, 5, padded)


def test_plan_groups_pairs_stably_by_owner():
    from bigrig_b200.ep import ExpertParallel
    ep = ExpertParallel.__new__(ExpertParallel)
    ep.world, ep.rank, ep.n_experts, ep.per_rank, ep.group = 4, 0, 16, 4, None
    idx = torch.tensor([[15, 0], [5, 4], [1, 14]], dtype=torch.int32)
    p = ep.plan(idx)
    assert p["order"].tolist() == [1, 4, 2, 3, 0, 5]
    assert p["dest"].tolist() == [0, 0, 1, 1, 3, 3]
    assert p["local"].tolist() == [0, 1, 1, 0, 3, 2]
    assert p["counts"].tolist() == [2, 2, 0, 2]
