"""Host side of the peer-memory expert-parallel group across 2 and 4 CPU ranks over gloo:
every rank allocates its buffer, the IPC handles travel over the process group, each rank
opens every other rank's and lists all of them in rank order (its own as allocated), and
closing unmaps the others' before freeing its own.  The library is a stand-in that
records the calls (the kernels themselves need GPUs: tests/test_gpu_peer.py and the
bench's multi-GPU check)."""
import ctypes
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

BASE = 0x10_0000_0000


class _FakeLib:
    def __init__(self, rank):
        self.rank, self.calls = rank, []

    def bigrig_peer_buffer_bytes(self, world, tokens, hidden, top_k):
        return 4096 * world

    def bigrig_peer_alloc(self, nbytes, ptr_ref, handle):
        ptr_ref._obj.value = BASE * (self.rank + 1)
        handle[0] = 0xB2
        handle[1] = self.rank                     # a handle names its owner
        self.calls.append(("alloc", nbytes))
        return 0

    def bigrig_peer_open(self, handle, ptr_ref):
        assert handle[0] == 0xB2 and handle[1] != self.rank, "own handle opened"
        ptr_ref._obj.value = BASE * (handle[1] + 1) + 0x100   # mapped elsewhere here
        self.calls.append(("open", handle[1]))
        return 0

    def bigrig_peer_close(self, ptr):
        self.calls.append(("close", ptr))
        return 0

    def bigrig_peer_free(self, ptr):
        self.calls.append(("free", ptr))
        return 0


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from bigrig_b200.ep import PeerBuffers
        lib = _FakeLib(rank)
        peers = PeerBuffers(1, 2048, 8, "cpu", wait_ms=250, lib=lib)
        c = peers.c
        bases = [c.base[i] for i in range(world)]
        fields = (c.world, c.rank, c.tokens, c.hidden, c.top_k, c.wait_ms)
        peers.close()
        q.put((rank, bases, fields, lib.calls))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_peer_group_maps_every_rank(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, bases, fields, calls in got:
        assert fields == (world, rank, 1, 2048, 8, 250)
        want = [BASE * (r + 1) + (0 if r == rank else 0x100) for r in range(world)]
        assert bases == want
        assert calls[0] == ("alloc", 4096 * world)
        opened = [c[1] for c in calls if c[0] == "open"]
        assert opened == [r for r in range(world) if r != rank]
        closed = [c[1] for c in calls if c[0] == "close"]
        assert closed == [BASE * (r + 1) + 0x100 for r in range(world) if r != rank]
        assert calls[-1] == ("free", BASE * (rank + 1))
