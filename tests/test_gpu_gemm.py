"""The tcgen05 grouped GEMM (prefill path) against the restatement of a multi-row
quantized matmul: weights dequantised into operand tiles (fp16 for fp16-scaled 4-bit
formats, as mx.dequantize gives them; bf16 otherwise), fp32 accumulation, the
activation h stored in the same type, bf16 output."""
import numpy as np
import pytest
import torch

from oracle import affine
from bigrig_b200 import _lib, ops
from tests._experts import Layer, assert_close, bf16_tensor, random_routing, to_f32

pytestmark = pytest.mark.gpu


@pytest.fixture
def path():
    prev = _lib.set_path("gemm")
    yield
    _lib.set_path(prev)


def _skewed(T, k, E, rng, skew=1.5):
    bias = rng.standard_normal(E) * skew
    lg = rng.standard_normal((T, E)) + bias
    return np.argsort(-lg, axis=1, kind="stable")[:, :k].astype(np.int32)


GEMM_CASES = [
    # H, I, E, k, bits, scale dtype, T       (mean rows per expert -> token tile)
    (1024, 512, 16, 4, 4, "float16", 64),     # 16 -> 32
    (2048, 768, 32, 8, 4, "bfloat16", 128),   # 32 -> 32, Qwen3 widths
    (512, 1024, 8, 2, 8, "float16", 512),     # 128 -> 128, 8-bit
    (2880, 2880, 8, 4, 4, "bfloat16", 256),   # 128 -> 128, partial 128-row feature tiles
    (1024, 512, 4, 2, 4, "float16", 1024),    # 512 -> 256, several token tiles per expert
    (768, 256, 16, 4, 4, "float16", 96),      # 24 -> 32, skewed: some experts empty
]


@pytest.mark.parametrize("H,I,E,k,bits,sd,T", GEMM_CASES)
def test_gemm_matches_oracle(cuda, path, H, I, E, k, bits, sd, T):
    rng = np.random.default_rng(H * 7 + T)
    L = Layer(H, I, E, bits, sd, seed=T + 1, slot_order=rng.permutation(E))
    x = affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    idx = _skewed(T, k, E, rng)
    n0 = _lib.launch_counts()["gemm_gate_up"]
    y = ops.switch_glu(bf16_tensor(x), torch.from_numpy(idx).to(cuda), L.slab, L.layout, E,
                       g2s=L.g2s)
    torch.cuda.synchronize()
    assert _lib.launch_counts()["gemm_gate_up"] == n0 + 1, "the GEMM path did not run"
    wr, inter = L.gemm_rounding()
    assert_close(to_f32(y), L.oracle_switch(x, idx, weight_round=wr, intermediate=inter))


def test_gemm_agrees_with_gemv(cuda):
    rng = np.random.default_rng(2)
    H, I, E, k, T = 1024, 512, 16, 4, 48
    L = Layer(H, I, E, 4, "float16", seed=9)
    xt = bf16_tensor(affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32)))
    it = torch.from_numpy(random_routing(T, k, E, rng)).to(cuda)
    prev = _lib.set_path("gemm")
    try:
        yg = ops.switch_glu(xt, it, L.slab, L.layout, E).clone()
        _lib.set_path("gemv")
        yv = ops.switch_glu(xt, it, L.slab, L.layout, E).clone()
    finally:
        _lib.set_path(prev)
    assert_close(to_f32(yg), to_f32(yv))


def test_gemm_batch_invariance(cuda, path):
    """A token's outputs do not depend on which other tokens share its experts' tiles."""
    rng = np.random.default_rng(4)
    H, I, E, k, T = 512, 256, 8, 2, 200
    L = Layer(H, I, E, 4, "bfloat16", seed=4)
    xt = bf16_tensor(affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32)))
    it = torch.from_numpy(random_routing(T, k, E, rng)).to(cuda)
    y = ops.switch_glu(xt, it, L.slab, L.layout, E)
    y2 = ops.switch_glu(xt.flip(0).contiguous(), it.flip(0).contiguous(), L.slab, L.layout, E)
    assert torch.equal(y, y2.flip(0))


def test_token_wise_prefill_matches_chunked(cuda):
    """A resident MoE stack prefilled layer-major in chunks and token-wise (each layer once
    over every chunk's tokens) gives the same bits: routing, the grouped GEMM's columns and
    the combine are all per token."""
    from bigrig_b200 import layered, stream
    from bigrig_b200.block import fill_store, make_blocks
    from bigrig_b200.fetch import HostExpertStore
    from bigrig_b200.formats import bytes_per_expert, make_spec
    LAYERS, H, I, E, K = 2, 1024, 512, 32, 8
    blocks = make_blocks(LAYERS, H, I, E, K, "olmoe", 4, 64, "float16", True, seed=5,
                         device=cuda)
    spec = make_spec(H, I, 4, 64, "float16")
    store = HostExpertStore({li: (E, bytes_per_expert(spec)) for li in range(LAYERS)})
    fill_store(store, LAYERS, H, I, E, 4, 64, "float16", seed=6, device=cuda)
    handle = stream.attach(blocks, store, E, policy="lfuda", warm="auto", device=cuda)
    g = torch.Generator(device=cuda)
    g.manual_seed(1)
    prompt = (torch.randn(600, H, generator=g, device=cuda) * 0.5).bfloat16()
    layers = [(lambda h, b=b: b(h, residual=h)) for b in blocks]
    n0 = _lib.launch_counts()["gemm_gate_up"]
    chunked = layered.prefill(layers, layered.chunks(prompt, 128))
    tw = layered.prefill(layers, layered.chunks(prompt, 128), token_wise=True)
    torch.cuda.synchronize()
    assert _lib.launch_counts()["gemm_gate_up"] == n0 + LAYERS * 5 + LAYERS
    del handle
    assert [c.shape[0] for c in tw] == [128, 128, 128, 128, 88]
    for a, b in zip(chunked, tw):
        assert torch.equal(a, b)
