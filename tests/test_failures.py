"""Failure paths, made on the host or by a bounded wait that runs out -- never by a fault.

* A fetch that fails in the middle of a step (the reference's fetch-failure cases,
  tests/test_fast_decode.py:355-501, moved to this design's host store): the error
  reaches the caller, the pool's tables stay consistent with its slab, and the next
  step with a working fetcher serves the same token.
* A closed fetcher is an error, not a silent miss.
* An expert-parallel rank that leaves before a layer's exchange: the other rank's
  collective ends with an error within the process group's short timeout (gloo, CPU).
* On the GPU, the persistent kernel's grid barrier made to wait for a CTA that does not
  exist: every CTA's bounded wait runs out and is counted in the error word, the kernel
  returns, and the next launch on the same context is correct.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

from bigrig_b200.fetch import HostExpertStore
from bigrig_b200.formats import make_spec
from bigrig_b200.stream import ExpertPool, StreamingSwitchGLU

SPEC = make_spec(64, 64, 4, 64, "float16")
BPE = sum(c["nbytes"] for p in SPEC.values() for c in p.values())


class FlakyStore(HostExpertStore):
    """A host store whose fetch raises OSError on the chosen call numbers."""

    def __init__(self, E, fail_on=()):
        super().__init__({0: (E, BPE)}, pin=False)
        for e in range(E):
            self.layers[0][e].fill_(e % 251)
        self.calls = 0
        self.fail_on = set(fail_on)

    def fetch(self, keys):
        self.calls += 1
        if self.calls in self.fail_on:
            raise OSError(f"injected read failure on fetch call {self.calls}")
        return super().fetch(keys)

    fetch_local = fetch


def _consistent(pool):
    g2s, s2g = pool.g2s, pool.s2g
    for e, s in enumerate(g2s):
        if s >= 0:
            assert s2g[s] == e
            assert torch.all(pool.slab[s, :pool.layout.bytes_per_expert] == e % 251)
    for s, e in enumerate(s2g):
        if e >= 0:
            assert g2s[e] == s


def test_fetch_failure_leaves_the_pool_consistent():
    E, C = 32, 8
    store = FlakyStore(E, fail_on={3})
    pool = ExpertPool(0, None, E, C, SPEC, device="cpu").build()
    mod = StreamingSwitchGLU(pool, store)
    rng = np.random.default_rng(4)
    toks = [rng.choice(E, 4, replace=False)[None] for _ in range(6)]
    for t in toks[:2]:
        mod.ensure(t)
    resident_before = set(np.flatnonzero(pool.g2s >= 0).tolist())
    with pytest.raises(OSError, match="injected"):
        mod.ensure(toks[2])
    _consistent(pool)
    # whatever the failed step could not fetch is not resident; nothing else was lost
    # beyond the slots freed for it
    assert set(np.flatnonzero(pool.g2s >= 0).tolist()) <= resident_before
    # the same token again, fetcher healthy: served, tables and bytes right
    slots = mod.ensure(toks[2])
    assert np.all(slots >= 0)
    _consistent(pool)
    for t in toks[3:]:
        mod.ensure(t)
        _consistent(pool)


def test_closed_fetcher_is_an_error():
    E, C = 16, 4
    store = FlakyStore(E)
    pool = ExpertPool(0, None, E, C, SPEC, device="cpu").build()
    mod = StreamingSwitchGLU(pool, store)
    store.close()
    with pytest.raises(RuntimeError, match="closed"):
        mod.ensure(np.array([[1, 2]]))


def _leaver(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    from bigrig_b200.ep import ExpertParallel
    ep = ExpertParallel(4)
    x = torch.randn(2, 8)
    idx = torch.tensor([[0, 3], [1, 2]], dtype=torch.int32)
    sc = torch.full((2, 2), 0.5)
    fn = lambda rows, ids: rows                                   # noqa: E731
    ep.dispatch_combine(x, idx, sc, fn, padded=True)               # one healthy layer
    def report(msg):
        q.put((rank, msg))
        q.close()
        q.join_thread()                                            # flushed before the exit

    if rank == 1:
        report("left")
        os._exit(0)                                                # leaves between steps
    try:
        ep.dispatch_combine(x, idx, sc, fn, padded=True)
        report("no error")
    except Exception as e:                                         # noqa: BLE001
        report(f"error: {type(e).__name__}")
    os._exit(0)


def test_peer_rank_leaving_ends_the_next_exchange_with_an_error():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res[1] == "left"
    assert res[0].startswith("error"), res


@pytest.mark.gpu
@pytest.mark.parametrize("path,kern", [("tiled", "decode_layer"), ("split", "decode_split")])
def test_persistent_kernel_barrier_timeout_is_reported(cuda, path, kern):
    from bigrig_b200 import _lib, ops
    from tests.test_gpu_decode_layer import SHAPES, _layer, _run, _words
    name = "olmoe"
    L, slab, g2s, x, gw, gb = _layer(name, cuda)
    ws = ops.Workspace(cuda)
    good, _, _ = _run(path, name, L, slab, g2s, x, gw, gb, ws)
    w0 = _words(ws)
    assert w0[1] == 0
    lib = _lib.load()
    n0 = _lib.launch_counts()[kern]
    assert lib.bigrig_test_grid_barrier(1, 1 << 14) == 0
    try:
        _run(path, name, L, slab, g2s, x, gw, gb, ws)
        torch.cuda.synchronize()
    finally:
        assert lib.bigrig_test_grid_barrier(0, 0) == 0
    assert _lib.launch_counts()[kern] == n0 + 1
    w1 = _words(ws)
    # every CTA's barrier wait ran out and said so
    assert w1[1] >= torch.cuda.get_device_properties(cuda).multi_processor_count, w1
    # the context is still usable and the next launch is right
    again, _, _ = _run(path, name, L, slab, g2s, x, gw, gb, ws)
    assert torch.equal(again, good)
    assert _words(ws)[1] == w1[1]
