"""The expert shapes beyond the gated SwiGLU expert, through the CUDA kernels.

The case matrix is the reference's (tests/test_fast_decode.py:95-110): the gated and
the plain (fc1/fc2, stream.py:48-76) projection layouts, each with and without the
affine projection ``bias`` (stream.py:79-81), and a spec that lists its components in
another order.  Added here: gpt-oss's clamped SwiGLU (a gated expert with biases, as
gpt-oss ships) and the squared ReLU of plain experts.  Every case runs the decode GEMV
chain, the tcgen05 grouped GEMM and a one-token layer (the persistent kernel takes
only the plain gated expert, so these run the three-kernel chain), each against the
numpy restatement with the same rounding points."""
import numpy as np
import pytest
import torch

from oracle import affine, moe, router
from bigrig_b200 import _lib, ops
from tests._experts import (Layer, assert_close, bf16_tensor, random_routing, report,
                            exceedance, to_f32)

pytestmark = pytest.mark.gpu

ORDER = ("biases", "bias", "scales", "weight")
CASES = {
    # name: Layer keyword arguments
    "gated": dict(),
    "plain": dict(plain=True),
    "gated+bias": dict(bias=True),
    "plain+bias": dict(plain=True, bias=True),
    "gated+bias, components biases/bias/scales/weight": dict(bias=True, order=ORDER),
    "gpt-oss act + bias": dict(bias=True, activation="gpt_oss"),
    "plain relu2 + f16 bias": dict(plain=True, bias=True, bias_dtype="float16", activation="relu2"),
    "gated + f32 bias, 8-bit": dict(bias=True, bias_dtype="float32", bits=8, scale_dtype="bfloat16"),
}


def _layer(name, H=512, I=256, E=16, seed=0):
    kw = dict(CASES[name])
    bits = kw.pop("bits", 4)
    sd = kw.pop("scale_dtype", "float16")
    rng = np.random.default_rng(seed + 11)
    return Layer(H, I, E, bits, sd, seed=seed, slot_order=rng.permutation(E), **kw)


@pytest.fixture
def path_mode():
    prev = _lib.set_path("auto")
    yield _lib.set_path
    _lib.set_path(prev)


@pytest.mark.parametrize("name", list(CASES))
def test_variant_gemv(cuda, path_mode, name):
    L = _layer(name)
    rng = np.random.default_rng(3)
    T, k = 3, 4
    x = affine.bf16_round(rng.standard_normal((T, L.H)).astype(np.float32))
    idx = random_routing(T, k, L.E, rng)
    path_mode("gemv")
    y = ops.switch_glu(bf16_tensor(x), torch.from_numpy(idx).to(cuda), L.slab, L.layout, L.E,
                       g2s=L.g2s)
    torch.cuda.synchronize()
    want = L.oracle_switch(x, idx)
    report(f"variant[{name}]-gemv", "kernel vs oracle", exceedance(to_f32(y), want))
    assert_close(to_f32(y), want)


@pytest.mark.parametrize("name", list(CASES))
def test_variant_gemm(cuda, path_mode, name):
    L = _layer(name, H=1024, I=512, seed=1)
    rng = np.random.default_rng(4)
    T, k = 64, 4
    x = affine.bf16_round(rng.standard_normal((T, L.H)).astype(np.float32))
    idx = random_routing(T, k, L.E, rng)
    path_mode("gemm")
    n0 = _lib.launch_counts()["gemm_gate_up"]
    y = ops.switch_glu(bf16_tensor(x), torch.from_numpy(idx).to(cuda), L.slab, L.layout, L.E,
                       g2s=L.g2s)
    torch.cuda.synchronize()
    assert _lib.launch_counts()["gemm_gate_up"] == n0 + 1, "the GEMM path did not run"
    wr, inter = L.gemm_rounding()
    want = L.oracle_switch(x, idx, weight_round=wr, intermediate=inter)
    report(f"variant[{name}]-gemm", "kernel vs oracle", exceedance(to_f32(y), want))
    assert_close(to_f32(y), want)


@pytest.mark.parametrize("name", ["plain+bias", "gpt-oss act + bias"])
def test_variant_one_token_layer(cuda, path_mode, name):
    """A one-token MoE layer from hidden states (router, experts, combine, residual)."""
    L = _layer(name, H=1024, I=512, E=32, seed=2)
    rng = np.random.default_rng(5)
    k = 4
    x = affine.bf16_round(rng.standard_normal((1, L.H)).astype(np.float32))
    gw = affine.bf16_round((rng.standard_normal((L.E, L.H)) * 0.02).astype(np.float32))
    gb = rng.standard_normal(L.E).astype(np.float32)
    xt, gwt = bf16_tensor(x), bf16_tensor(gw)
    out, idx, sc = ops.moe_layer(xt, gwt, torch.from_numpy(gb).to(cuda), k, L.slab, L.layout,
                                 L.E, "topk_softmax", False, g2s=L.g2s, residual=xt)
    torch.cuda.synchronize()
    logits = (x @ gw.T + gb).astype(np.float32)
    widx, _ = router.topk(logits, k, mode="topk_softmax")
    np.testing.assert_array_equal(np.sort(idx.cpu().numpy(), axis=1), np.sort(widx, axis=1))
    comb = moe.combine(L.oracle_switch(x, idx.cpu().numpy()), sc.cpu().numpy())
    want = affine.bf16_round(x + comb)
    assert_close(to_f32(out), want)


def test_plain_dequant_refuses_projection_one(cuda):
    L = _layer("plain")
    with pytest.raises(ValueError):
        ops.dequant(L.slab, L.layout, 0, 1)
    # fc1 and fc2 dequantise bit-exactly like any projection
    for proj, name in ((0, "fc1"), (2, "fc2")):
        got = ops.dequant(L.slab, L.layout, int(L.slot_of[5]), proj).float().cpu().numpy()
        codes, s, b = L.q[5][name]
        want = affine.dequantize(codes, s, b, 64, L.bits, L.sd)
        np.testing.assert_array_equal(got, affine.half_bits_to_f32(want, L.sd)
                                      if want.dtype == np.uint16 else want)
