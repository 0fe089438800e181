"""The peer-memory expert-parallel layer (bigrig_peer_layer) on one GPU: a group of one
rank is its own peer, so gather, route, experts, scatter and combine all run, the flags
included, and the result must equal the same layer computed by the library's separate
calls (router, switch_glu, combine) bit for bit, eagerly and replayed from a CUDA graph.
A group whose second rank is never there makes the bounded waits run out: the layer
finishes and the error word says so.  Multi-rank runs are checked by bench.py's
expert-parallel check against one GPU holding every expert."""
import ctypes

import numpy as np
import pytest
import torch

from bigrig_b200 import _lib, ops
from bigrig_b200.ep import PeerBuffers
from tests._experts import Layer, bf16_tensor

pytestmark = pytest.mark.gpu


def _reference(L, x, gw, gb, k, mode, norm, residual):
    idx, sc = ops.router_topk(ops.router_logits(x, gw, gb), k, mode, norm)
    y = ops.switch_glu(x, idx, L.slab, L.layout, L.E, g2s=L.g2s)
    return ops.combine(y, sc, residual=residual)


@pytest.mark.parametrize("T,H,I,E,k,mode,norm", [
    (1, 2048, 1024, 64, 8, "softmax_topk", False),    # OLMoE-shaped decode token
    (4, 1024, 512, 32, 8, "softmax_topk", True),      # 32 pairs: the GEMV chain's limit
    (8, 512, 256, 16, 4, "topk_softmax", False),      # 32 pairs
    (6, 1024, 256, 32, 8, "topk_softmax", False),     # 48 pairs: grouped GEMM path
])
def test_peer_layer_matches_separate_calls(cuda, T, H, I, E, k, mode, norm):
    L = Layer(H, I, E, 4, "float16", seed=H + E)
    rng = np.random.default_rng(T * 7 + E)
    gw = bf16_tensor((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
    gb = torch.from_numpy(rng.standard_normal(E).astype(np.float32)).to(cuda)
    peers = PeerBuffers(T, H, k, cuda)
    try:
        n0 = _lib.launch_counts()
        for step in range(3):                      # each call advances the flags' count
            x = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32))
            res = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32))
            got = ops.peer_layer(peers, x, gw, gb, E, 0, E, L.slab, L.layout, mode, norm,
                                 g2s=L.g2s, residual=res)
            want = _reference(L, x, gw, gb, k, mode, norm, res)
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"step {step}"
        n1 = _lib.launch_counts()
        for name in ("peer_gather", "peer_scatter", "peer_combine"):
            assert n1[name] - n0[name] == 3, name
        # decode-sized calls route in one launch (the chain's route kernel), larger ones
        # localize the separately routed ids
        key = "route" if T * k <= 32 else "peer_localize"
        assert n1[key] - n0[key] == 3, key
        assert peers.errors() == 0
    finally:
        peers.close()


def test_peer_layer_in_a_cuda_graph(cuda):
    T, H, I, E, k = 1, 2048, 1024, 64, 8
    L = Layer(H, I, E, 4, "float16", seed=11)
    rng = np.random.default_rng(5)
    gws = [bf16_tensor((rng.standard_normal((E, H)) * 0.02).astype(np.float32)) for _ in range(3)]
    peers = PeerBuffers(T, H, k, cuda)
    ws = ops.Workspace(cuda)
    ws.reserve(ops.peer_workspace_bytes(peers, E, E, L.layout))
    try:
        xin = torch.zeros(T, H, dtype=torch.bfloat16, device=cuda)

        def stack(x):
            h = x
            for gw in gws:
                h = ops.peer_layer(peers, h, gw, None, E, 0, E, L.slab, L.layout, g2s=L.g2s,
                                   residual=h, workspace=ws)
            return h

        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            stack(xin)
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            yout = stack(xin)
        for step in range(3):
            x = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32))
            xin.copy_(x)
            g.replay()
            h = x
            for gw in gws:
                h = _reference(L, h, gw, None, k, "softmax_topk", False, h)
            torch.cuda.synchronize()
            assert torch.equal(yout.view(torch.int16), h.view(torch.int16)), f"replay {step}"
        del g
        assert peers.errors() == 0
    finally:
        peers.close()


def test_peer_wait_runs_out_on_a_missing_rank(cuda):
    """A group of two whose 'other rank' is this process's own buffer under a second name:
    nobody raises the flags rank 1 would, so the gather's wait runs out (its bound set to
    0.2 s), the layer still finishes, the error word counts it, and later waits return at
    once."""
    T, H, I, E, k = 1, 512, 256, 16, 4
    L = Layer(H, I, E, 4, "float16", seed=3)
    lib = _lib.load()
    nbytes = lib.bigrig_peer_buffer_bytes(2, T, H, k)
    own = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * _lib.PEER_HANDLE_BYTES)()
    _lib.check(lib.bigrig_peer_alloc(nbytes, ctypes.byref(own), handle), "peer_alloc")
    try:
        g = _lib.PeerGroup(world=2, rank=0, tokens=T, hidden=H, top_k=k, wait_ms=200)
        g.base[0] = own.value
        g.base[1] = own.value

        class _Group:                                  # ops.peer_layer's view of a group
            c, tokens, hidden = g, T, H

        rng = np.random.default_rng(9)
        gw = bf16_tensor((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
        x = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32))
        ops.peer_layer(_Group, x, gw, None, E, 0, E, L.slab, L.layout, g2s=L.g2s)
        ops.peer_layer(_Group, x, gw, None, E, 0, E, L.slab, L.layout, g2s=L.g2s)
        torch.cuda.synchronize()
        n = ctypes.c_int32(0)
        _lib.check(lib.bigrig_peer_errors(ctypes.byref(g), ctypes.byref(n), None), "peer_errors")
        assert n.value == 1                            # one wait ran out; the rest returned
        _lib.check(lib.bigrig_peer_errors(ctypes.byref(g), ctypes.byref(n), None), "peer_errors")
        assert n.value == 0
    finally:
        torch.cuda.synchronize()
        lib.bigrig_peer_free(own)


def test_peer_layer_shares_a_workspace_with_the_one_token_kernel(cuda):
    """Peer layers and the persistent one-token layer kernel on one workspace, interleaved:
    the one-token kernel keeps its barrier counter and error words at the head of every
    workspace, and the peer layer must leave them as it found them."""
    T, H, I, E, k = 1, 2048, 1024, 64, 8
    L = Layer(H, I, E, 4, "float16", seed=21)
    rng = np.random.default_rng(21)
    gw = bf16_tensor((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
    gb = torch.from_numpy(rng.standard_normal(E).astype(np.float32)).to(cuda)
    peers = PeerBuffers(T, H, k, cuda)
    ws = ops.Workspace(cuda)
    try:
        xs = [bf16_tensor(rng.standard_normal((T, H)).astype(np.float32)) for _ in range(4)]
        want = [ops.moe_layer(x, gw, gb, k, L.slab, L.layout, E, g2s=L.g2s, residual=x,
                              workspace=ops.Workspace(cuda))[0] for x in xs]
        n0 = _lib.launch_counts()
        for x, w in zip(xs, want):
            p = ops.peer_layer(peers, x, gw, gb, E, 0, E, L.slab, L.layout, g2s=L.g2s,
                               residual=x, workspace=ws)
            got = ops.moe_layer(x, gw, gb, k, L.slab, L.layout, E, g2s=L.g2s, residual=x,
                                workspace=ws)[0]
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int16), w.view(torch.int16))
            assert torch.equal(p.view(torch.int16),
                               _reference(L, x, gw, gb, k, "softmax_topk", False, x).view(torch.int16))
        n1 = _lib.launch_counts()
        assert n1["decode_layer"] + n1["decode_split"] - n0["decode_layer"] - n0["decode_split"] == 4
        assert ws.errors() == 0 and peers.errors() == 0
    finally:
        peers.close()


def test_peer_layer_gemv_past_the_fused_route(cuda):
    """More than 32 pairs on the GEMV pair (what a large group's per-rank share takes):
    routed, localised and permuted in separate launches, then the same GEMV kernels as
    switch_glu under the same path."""
    T, H, I, E, k = 6, 1024, 256, 32, 8
    L = Layer(H, I, E, 4, "float16", seed=33)
    rng = np.random.default_rng(33)
    gw = bf16_tensor((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
    peers = PeerBuffers(T, H, k, cuda)
    old = _lib.set_path("gemv")
    try:
        for step in range(2):
            x = bf16_tensor(rng.standard_normal((T, H)).astype(np.float32))
            n0 = _lib.launch_counts()
            got = ops.peer_layer(peers, x, gw, None, E, 0, E, L.slab, L.layout, g2s=L.g2s,
                                 residual=x)
            n1 = _lib.launch_counts()
            want = _reference(L, x, gw, None, k, "softmax_topk", False, x)
            torch.cuda.synchronize()
            assert torch.equal(got.view(torch.int16), want.view(torch.int16)), f"step {step}"
            assert n1["peer_localize"] - n0["peer_localize"] == 1
            assert n1["gate_up"] - n0["gate_up"] == 1 and n1["gemm_gate_up"] == n0["gemm_gate_up"]
        assert peers.errors() == 0
    finally:
        _lib.set_path(old)
        peers.close()
