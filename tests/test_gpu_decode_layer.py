"""The persistent one-token decode kernels (one cooperative launch per MoE layer): the
feature-tiled kernel (path "tiled") and the split kernel (path "split": units of one
routed expert's 64 intermediate features, integer tensor-core dot products); AUTO takes the
split kernel for layers whose units fill two waves of SMs (the Mixtral shape), else tiled.

Its routing must be the three-kernel chain's bit for bit (indices and scores); its
output, computed on the tensor cores in another summation order, must meet the expert
parity bar against the chain and against exact fp32 weights in plain torch -- at the full
layer sizes of every family it runs, with and without the residual, for 4- and 8-bit
codes, one to eight routed experts and a missing slot.  It must give the same bits on
every call (its flag words carry over between launches), count no error and no wait
timeout, and replay the same bits from a CUDA graph.
"""
import numpy as np
import pytest
import torch

from bigrig_b200 import _lib, formats, ops
from bigrig_b200.block import random_expert_bytes
from tests._experts import assert_close, exceedance, report
from tests.test_gpu_fullsize import CONFIGS, _dequant_f32

pytestmark = pytest.mark.gpu

torch.backends.cuda.matmul.allow_tf32 = False

SHAPES = {
    # name: H, I, E, k, bits, scale dtype, mode, norm_topk
    "olmoe": CONFIGS["olmoe"] + ("softmax_topk", False),
    "qwen3": CONFIGS["qwen3"] + ("softmax_topk", True),
    "gpt_oss": CONFIGS["gpt_oss"] + ("topk_softmax", False),
    "olmoe_8bit": (2048, 1024, 64, 8, 8, "bfloat16", "softmax_topk", False),
    "k2": (1024, 512, 32, 2, 4, "float16", "topk_softmax", False),
    "k1": (512, 256, 16, 1, 4, "float16", "softmax_topk", False),
    "mixtral": CONFIGS["mixtral"] + ("topk_softmax", False),   # too wide for "tiled"
}
TILED_TOO_WIDE = {"mixtral"}
AUTO_SPLIT = {"mixtral"}          # k * I / 64 >= 2 x 148 units


def _layer(name, device):
    H, I, E, k, bits, sd, mode, norm = SHAPES[name]
    spec = formats.make_spec(H, I, bits, 64, sd)
    L = formats.layout_from_spec(spec, {"bits": bits, "group_size": 64, "mode": "affine"})
    g = torch.Generator(device=device)
    g.manual_seed(sum(map(ord, name)) + 7)
    slab = torch.zeros(E, L.slot_stride, dtype=torch.uint8, device=device)
    tdt = torch.float16 if sd == "float16" else torch.bfloat16
    for e in range(E):
        slab[e, :L.bytes_per_expert] = random_expert_bytes(H, I, bits, 64, tdt, g, device)
    perm = torch.from_numpy(np.random.default_rng(E).permutation(E)).to(device)
    slab = slab[perm].contiguous()                  # expert e lives in slot g2s[e]
    g2s = torch.argsort(perm).to(torch.int32)
    x = (torch.randn(1, H, generator=g, device=device) * 0.5).bfloat16()
    gw = (torch.randn(E, H, generator=g, device=device) * 0.05).bfloat16()
    gb = torch.randn(E, generator=g, device=device) * 0.1
    return L, slab, g2s, x, gw, gb


def _words(ws):
    """The workspace's error and synchronisation words (int32 [8])."""
    torch.cuda.synchronize()
    return ws.buf[:32].view(torch.int32).cpu().numpy().copy()


def _run(path, name, L, slab, g2s, x, gw, gb, ws, residual=None):
    H, I, E, k, bits, sd, mode, norm = SHAPES[name]
    prev = _lib.set_path(path)
    try:
        return ops.moe_layer(x, gw, gb, k, slab, L, E, mode, norm, g2s=g2s, residual=residual,
                             workspace=ws)
    finally:
        _lib.set_path(prev)


@pytest.mark.parametrize("path", ["auto", "tiled", "split"])
@pytest.mark.parametrize("name", list(SHAPES))
def test_persistent_equals_chain(cuda, name, path):
    L, slab, g2s, x, gw, gb = _layer(name, cuda)
    ws = ops.Workspace(cuda)
    fits = path != "tiled" or name not in TILED_TOO_WIDE
    n0 = _lib.launch_counts()
    out, idx, sc = _run(path, name, L, slab, g2s, x, gw, gb, ws)
    out_r, idx_r, sc_r = _run(path, name, L, slab, g2s, x, gw, gb, ws, residual=x)
    n1 = _lib.launch_counts()
    split = path == "split" or (path == "auto" and name in AUTO_SPLIT)
    kern = "decode_split" if split else "decode_layer"
    assert n1[kern] - n0[kern] == (2 if fits else 0)
    if fits:
        assert n1["route"] == n0["route"]
    words = _words(ws)
    assert words[0] == 0 and words[1] == 0, words      # no errors, no wait timed out
    cout, cidx, csc = _run("chain", name, L, slab, g2s, x, gw, gb, ws)
    cout_r, _, _ = _run("chain", name, L, slab, g2s, x, gw, gb, ws, residual=x)
    assert torch.equal(idx, cidx) and torch.equal(sc, csc)
    assert torch.equal(idx_r, cidx) and torch.equal(sc_r, csc)
    assert_close(out.float().cpu().numpy(), cout.float().cpu().numpy())
    # the residual add, exactly: out = bf16(x + bf16(sum_j score_j y_j)) on the same sums
    # (the parity bar is for the expert output: after the add, a one-ulp difference in the
    # rounded sum is no longer small next to an output the residual nearly cancels)
    assert torch.equal(out_r, (x.float() + out.float()).bfloat16())
    assert torch.equal(cout_r, (x.float() + cout.float()).bfloat16())
    # consecutive calls reuse the same flag words: the same bits every time
    for _ in range(3):
        again, _, _ = _run(path, name, L, slab, g2s, x, gw, gb, ws)
        assert torch.equal(again, out)
    # against exact fp32 weights in plain torch, with the kernels' rounding points
    xf = x.float()
    ref = torch.zeros(L.hidden, dtype=torch.float32, device=cuda)
    for j in range(idx.shape[1]):
        slot = int(g2s[int(idx[0, j])])
        w = [_dequant_f32(slab, L, slot, p) for p in range(3)]
        h = (torch.nn.functional.silu(xf @ w[0].T) * (xf @ w[1].T)).bfloat16().float()
        y = (h @ w[2].T).bfloat16().float()
        ref += sc[0, j] * y[0]
    got, want = out.float().cpu().numpy()[0], ref.bfloat16().float().cpu().numpy()
    report(f"persistent_equals_chain[{name}-{path}]", "layer vs fp32", exceedance(got, want))
    assert_close(got, want)


def test_persistent_missing_slot(cuda):
    """A routed expert without a slot is counted and contributes zeros, as in the chain."""
    name = "olmoe"
    L, slab, g2s, x, gw, gb = _layer(name, cuda)
    ws = ops.Workspace(cuda)
    _, idx, _ = _run("auto", name, L, slab, g2s, x, gw, gb, ws)
    holes = g2s.clone()
    holes[idx[0, 0]] = -1
    holes[idx[0, 3]] = -1
    out, _, _ = _run("auto", name, L, slab, holes, x, gw, gb, ws)
    assert ws.errors() > 0
    cout, _, _ = _run("chain", name, L, slab, holes, x, gw, gb, ws)
    assert_close(out.float().cpu().numpy(), cout.float().cpu().numpy())
    full, _, _ = _run("auto", name, L, slab, g2s, x, gw, gb, ws)
    assert not torch.equal(out, full)
    ws.errors()
    words = _words(ws)
    assert words[1] == 0, words


def test_persistent_graph_replay(cuda):
    """Captured into a CUDA graph (a layer stack of four), replays give the eager bits."""
    name = "olmoe"
    L, slab, g2s, x, gw, gb = _layer(name, cuda)
    H, I, E, k, bits, sd, mode, norm = SHAPES[name]
    ws = ops.Workspace(cuda)
    ws.reserve(ops.workspace_bytes(1, k, E, L))
    hs = [x.clone() for _ in range(5)]
    idx = torch.empty(1, k, dtype=torch.int32, device=cuda)
    sc = torch.empty(1, k, dtype=torch.float32, device=cuda)

    def stack():
        for i in range(4):
            ops.moe_layer(hs[i], gw, gb, k, slab, L, E, mode, norm, g2s=g2s, residual=hs[i],
                          out=hs[i + 1], indices=idx, scores=sc, workspace=ws)

    stack()
    want = hs[4].clone()
    s = torch.cuda.Stream(device=cuda)
    s.wait_stream(torch.cuda.current_stream(cuda))
    with torch.cuda.stream(s):
        stack()
    torch.cuda.current_stream(cuda).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        stack()
    for _ in range(3):
        hs[4].zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(hs[4], want)
    del graph
    words = _words(ws)
    assert words[0] == 0 and words[1] == 0, words


@pytest.mark.parametrize("name", list(SHAPES))
def test_routed_layer_equals_routing_layer(cuda, name):
    """bigrig_moe_layer_routed on the routing bigrig_moe_layer computed gives its bits, with
    and without the residual (the persistent kernel without its router phase, or for the
    too-wide layer the expert chain plus combine), and counts no error."""
    H, I, E, k, bits, sd, mode, norm = SHAPES[name]
    L, slab, g2s, x, gw, gb = _layer(name, cuda)
    ws = ops.Workspace(cuda)
    for residual in (None, x):
        out, idx, sc = _run("auto", name, L, slab, g2s, x, gw, gb, ws, residual=residual)
        n0 = _lib.launch_counts()
        got = ops.moe_layer_routed(x, idx, sc, slab, L, E, g2s=g2s, residual=residual, workspace=ws)
        n1 = _lib.launch_counts()
        assert torch.equal(got, out)
        assert n1["router_logits"] == n0["router_logits"] and n1["route"] == n0["route"]
    assert ws.errors() == 0
    assert _words(ws)[1] == 0


def test_routed_layer_counts_missing_slots(cuda):
    name = "olmoe"
    H, I, E, k, bits, sd, mode, norm = SHAPES[name]
    L, slab, g2s, x, gw, gb = _layer(name, cuda)
    ws = ops.Workspace(cuda)
    out, idx, sc = _run("auto", name, L, slab, g2s, x, gw, gb, ws)
    holes = g2s.clone()
    holes[idx[0, 1]] = -1
    got = ops.moe_layer_routed(x, idx, sc, slab, L, E, g2s=holes, workspace=ws)
    want, _, _ = _run("chain", name, L, slab, holes, x, gw, gb, ws)
    assert ws.errors() > 0
    assert_close(got.float().cpu().numpy(), want.float().cpu().numpy())
