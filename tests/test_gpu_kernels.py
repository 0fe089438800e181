"""Parity of each sm_100a kernel with the CPU restatement, called through the C ABI.

Bar (north star): dequantised weights, routing indices and the permutation bit for
bit; expert outputs within 1e-2 relative / 2e-3 absolute (bf16).
"""
import numpy as np
import pytest
import torch

from oracle import affine, moe, router
from bigrig_b200 import _lib, ops
from tests._experts import Layer, assert_close, bf16_tensor, random_routing, to_f32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits,sd,H,I", [(4, "float16", 256, 128), (4, "bfloat16", 2880, 192),
                                         (8, "float16", 512, 256), (8, "bfloat16", 128, 448)])
def test_dequant_bit_exact(cuda, bits, sd, H, I):
    L = Layer(H, I, 3, bits, sd, seed=bits + H)
    for e in range(3):
        for proj, name in enumerate(moe.PROJ):
            got = ops.dequant(L.slab, L.layout, L.slot_of[e], proj)
            want = affine.dequantize(*L.q[e][name], 64, bits, sd)
            np.testing.assert_array_equal(got.view(torch.int16).cpu().numpy().view(np.uint16), want)


@pytest.mark.parametrize("T,H,E", [(1, 2048, 64), (37, 2048, 128), (5, 2880, 128), (3, 4096, 8)])
def test_router_logits(cuda, T, H, E):
    rng = np.random.default_rng(T + E)
    x = affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    w = affine.bf16_round((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
    b = rng.standard_normal(E).astype(np.float32)
    got = ops.router_logits(bf16_tensor(x), bf16_tensor(w), torch.from_numpy(b).to(cuda))
    want = router.router_logits(x, w, b)
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("mode,norm", [("softmax_topk", False), ("softmax_topk", True),
                                       ("topk_softmax", False)])
@pytest.mark.parametrize("T,E,k", [(1, 64, 8), (129, 128, 8), (64, 128, 4), (7, 8, 2),
                                   (33, 256, 8), (3, 40, 32), (2, 1, 1)])
def test_router_topk_exact(cuda, mode, norm, T, E, k):
    rng = np.random.default_rng(E * 31 + k)
    lg = (rng.standard_normal((T, E)) + rng.standard_normal(E)).astype(np.float32)
    idx, sc = ops.router_topk(torch.from_numpy(lg).to(cuda), k, mode, norm)
    widx, wsc = router.topk(lg, k, mode, norm)
    np.testing.assert_array_equal(idx.cpu().numpy(), widx)
    np.testing.assert_allclose(sc.cpu().numpy(), wsc, rtol=2e-6, atol=1e-7)


def test_router_topk_ties_and_bf16(cuda):
    rng = np.random.default_rng(9)
    lg = np.round(rng.standard_normal((200, 64)) * 2) / 2          # many exact ties
    lg = affine.bf16_round(lg.astype(np.float32))
    t = bf16_tensor(lg)
    for mode in ("softmax_topk", "topk_softmax"):
        idx, sc = ops.router_topk(t, 8, mode)
        widx, wsc = router.topk(lg, 8, mode)
        np.testing.assert_array_equal(idx.cpu().numpy(), widx)
        np.testing.assert_allclose(sc.cpu().numpy(), wsc, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("T,k,E", [(1, 8, 64), (128, 8, 64), (4096, 8, 128), (16384, 4, 128),
                                   (8192, 2, 8), (300, 8, 256), (50, 1, 3)])
def test_permutation_exact(cuda, T, k, E):
    rng = np.random.default_rng(T + k)
    idx = random_routing(T, k, E, rng) if k <= E else None
    got = ops.moe_permute(torch.from_numpy(idx).to(cuda), E)
    want = router.permutation(idx, E)
    for key in ("order", "inv", "offsets"):
        np.testing.assert_array_equal(got[key].cpu().numpy(), want[key], err_msg=key)
    ns = int(got["num_seg"].item())
    assert ns == len(want["seg_expert"])
    np.testing.assert_array_equal(got["seg_expert"].cpu().numpy()[:ns], want["seg_expert"])
    np.testing.assert_array_equal(got["seg_start"].cpu().numpy()[:ns + 1], want["seg_start"])
    assert int(got["err"].item()) == 0


def test_permutation_skewed_and_degenerate(cuda):
    # every pair on one expert, and a heavily skewed draw: stability is what is tested
    for idx in (np.zeros((1000, 1), np.int32),
                np.random.default_rng(1).zipf(1.3, size=(3000, 4)).clip(1, 64).astype(np.int32) - 1):
        got = ops.moe_permute(torch.from_numpy(np.ascontiguousarray(idx)).to(cuda), 64)
        want = router.permutation(idx, 64)
        np.testing.assert_array_equal(got["order"].cpu().numpy(), want["order"])
        np.testing.assert_array_equal(got["inv"].cpu().numpy(), want["inv"])


CASES = [
    # H, I, E, k, bits, scale dtype, T
    (2048, 1024, 64, 8, 4, "float16", 1),      # OLMoE decode
    (2048, 1024, 16, 8, 4, "float16", 3),
    (1024, 512, 32, 8, 4, "float16", 128),     # a prefill-sized call on the GEMV path
    (2048, 768, 16, 8, 4, "bfloat16", 8),      # Qwen3 shape, batch-8 decode
    (2880, 2880, 8, 4, 4, "bfloat16", 2),      # gpt-oss shape (K = 45 groups)
    (4096, 1024, 8, 2, 8, "float16", 1),       # 8-bit, wide hidden
    (256, 14336, 4, 2, 8, "float16", 5),       # Mixtral's 14336-wide down projection
]


@pytest.mark.parametrize("H,I,E,k,bits,sd,T", CASES)
def test_switch_glu_matches_oracle(cuda, H, I, E, k, bits, sd, T):
    rng = np.random.default_rng(H + I + T)
    L = Layer(H, I, E, bits, sd, seed=T, slot_order=rng.permutation(E))
    x = affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    idx = random_routing(T, k, E, rng)
    prev = _lib.set_path("gemv")
    try:
        y = ops.switch_glu(bf16_tensor(x), torch.from_numpy(idx).to(cuda), L.slab, L.layout, E,
                           g2s=L.g2s)
    finally:
        _lib.set_path(prev)
    assert_close(to_f32(y), L.oracle_switch(x, idx))


def test_moe_forward_equals_switch_then_combine(cuda):
    rng = np.random.default_rng(11)
    H, I, E, k, T = 1024, 512, 32, 8, 6
    L = Layer(H, I, E, 4, "float16", seed=3)
    x = affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    lg = (rng.standard_normal((T, E)) + rng.standard_normal(E)).astype(np.float32)
    xt, lt = bf16_tensor(x), torch.from_numpy(lg).to(cuda)
    out, idx, sc = ops.moe_forward(xt, lt, k, L.slab, L.layout, E, "softmax_topk", False)
    y = ops.switch_glu(xt, idx, L.slab, L.layout, E)
    ref = ops.combine(y, sc)
    assert torch.equal(out, ref)
    widx, wsc = router.topk(lg, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), widx)
    want = moe.combine(L.oracle_switch(x, widx), wsc)
    assert_close(to_f32(out), want)


def test_missing_slot_is_reported_not_read(cuda):
    H, I, E = 256, 128, 8
    L = Layer(H, I, E, 4, "float16", seed=5)
    g2s = L.g2s.clone()
    g2s[3] = -1
    x = bf16_tensor(np.ones((2, H), np.float32))
    idx = torch.tensor([[3, 1], [2, 3]], dtype=torch.int32, device=cuda)
    ws = ops.Workspace(cuda)
    y = ops.switch_glu(x, idx, L.slab, L.layout, E, g2s=g2s, workspace=ws)
    assert ws.errors() > 0
    yy = y.float().cpu().numpy()
    assert np.all(yy[0, 0] == 0) and np.all(yy[1, 1] == 0)
    assert np.any(yy[0, 1] != 0)
    assert ws.errors() == 0


@pytest.fixture
def chain_path():
    """One-token moe_layer calls on the three-kernel chain (not the persistent kernel)."""
    prev = _lib.set_path("chain")
    yield
    _lib.set_path(prev)


@pytest.mark.parametrize("T,k,E,mode", [(1, 8, 64, "softmax_topk"), (2, 8, 128, "softmax_topk"),
                                        (4, 4, 128, "topk_softmax"), (16, 2, 8, "topk_softmax")])
def test_fused_decode_layer_is_bit_identical(cuda, T, k, E, mode, chain_path):
    """The fused three-kernel decode chain (route, gate_up, down+combine) computes exactly
    what the separate kernels compute, with and without the residual."""
    rng = np.random.default_rng(T * 100 + E)
    H, I = 1024, 512
    L = Layer(H, I, E, 4, "float16", seed=T, slot_order=rng.permutation(E))
    x = bf16_tensor(affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32)))
    gw = bf16_tensor(affine.bf16_round((rng.standard_normal((E, H)) * 0.02).astype(np.float32)))
    gb = torch.from_numpy(rng.standard_normal(E).astype(np.float32)).to(cuda)
    out, idx, sc = ops.moe_layer(x, gw, gb, k, L.slab, L.layout, E, mode, False, g2s=L.g2s)
    out_r, _, _ = ops.moe_layer(x, gw, gb, k, L.slab, L.layout, E, mode, False, g2s=L.g2s,
                                residual=x)
    n0 = _lib.launch_counts()
    lg = ops.router_logits(x, gw, gb)
    idx2, sc2 = ops.router_topk(lg, k, mode)
    y = ops.switch_glu(x, idx2, L.slab, L.layout, E, g2s=L.g2s)
    ref = ops.combine(y, sc2)
    n1 = _lib.launch_counts()
    assert n1["route"] == n0["route"]
    assert torch.equal(idx, idx2) and torch.equal(sc, sc2)
    assert torch.equal(out, ref)
    assert torch.equal(out_r, (x.float() + ref.float()).bfloat16())
    lt = lg.clone()
    fo, fidx, fsc = ops.moe_forward(x, lt, k, L.slab, L.layout, E, mode, False, g2s=L.g2s)
    assert torch.equal(fo, ref) and torch.equal(fidx, idx2)
    widx, wsc = router.topk(lg.cpu().numpy(), k, mode)
    np.testing.assert_array_equal(idx.cpu().numpy(), widx)
    xf = to_f32(x)
    assert_close(to_f32(out), moe.combine(L.oracle_switch(xf, widx), wsc))
