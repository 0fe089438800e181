"""The pool on the GPU: a streamed layer's output is bit-identical to the same layer held
whole (the reference's core invariant, bigrig_engine/stream.py:25-31), on decode steps,
on a prompt that needs more experts than slots (expert-sorted spans), and through the
MoE block; the slab holds exactly the bytes the tables say."""
import numpy as np
import pytest
import torch

from oracle import affine
from bigrig_b200.block import MoEBlock
from bigrig_b200.fetch import HostExpertStore
from bigrig_b200.stream import ExpertPool, StreamHandle, StreamingSwitchGLU
from bigrig_b200 import _lib
from tests._experts import Layer, assert_close, bf16_tensor

pytestmark = pytest.mark.gpu

H, I, E, K = 1024, 512, 64, 8


@pytest.fixture(scope="module")
def layer(cuda):
    L = Layer(H, I, E, 4, "float16", seed=21)
    store = HostExpertStore({0: (E, L.layout.bytes_per_expert)}, pin=True)
    for e in range(E):
        store.put(0, e, L.blobs[e])
    return L, store


def _full(L, store, cuda):
    pool = ExpertPool(0, None, E, E, L.spec, device=cuda).build()
    mod = StreamingSwitchGLU(pool, store)
    StreamHandle(None, [pool], [mod], store).warm("auto")
    assert mod.refresh()
    return mod


def _skewed_routing(T, rng):
    bias = np.linspace(2.0, -2.0, E)
    lg = rng.standard_normal((T, E)) + bias
    return np.argsort(-lg, axis=1, kind="stable")[:, :K].astype(np.int32)


@pytest.mark.parametrize("C,policy", [(8, "lfuda"), (16, "lfuda"), (12, "lru"), (20, "s3fifo")])
def test_streamed_decode_is_bit_identical(layer, cuda, C, policy):
    L, store = layer
    full = _full(L, store, cuda)
    pool = ExpertPool(0, None, E, C, L.spec, policy=policy, device=cuda).build()
    mod = StreamingSwitchGLU(pool, store)
    rng = np.random.default_rng(C)
    routing = _skewed_routing(60, rng)
    for t in range(routing.shape[0]):
        x = bf16_tensor(affine.bf16_round(rng.standard_normal((1, H)).astype(np.float32)))
        idx = torch.from_numpy(routing[t:t + 1]).to(cuda)
        assert torch.equal(mod(x, idx), full(x, idx)), f"step {t}"
    assert pool.misses > C and pool.evicts > 0
    torch.cuda.synchronize()
    for slot, e in enumerate(pool.s2g):
        if e >= 0:
            assert torch.equal(pool.slab[slot, :L.layout.bytes_per_expert].cpu(), store.layers[0][e])


def test_streamed_prompt_spans_are_bit_identical(layer, cuda):
    L, store = layer
    full = _full(L, store, cuda)
    pool = ExpertPool(0, None, E, 8, L.spec, device=cuda).build()
    mod = StreamingSwitchGLU(pool, store)
    rng = np.random.default_rng(5)
    T = 24
    x = bf16_tensor(affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32)))
    idx = torch.from_numpy(_skewed_routing(T, rng)).to(cuda)
    assert len(np.unique(idx.cpu().numpy())) > 8
    y = mod(x.reshape(1, T, H), idx.reshape(1, T, K))
    assert mod.chunked_calls == 1
    assert y.shape == (1, T, K, H)
    assert torch.equal(y.reshape(T, K, H), full(x, idx))


def test_topk_above_capacity_raises(layer, cuda):
    L, store = layer
    pool = ExpertPool(0, None, E, 4, L.spec, device=cuda).build()
    mod = StreamingSwitchGLU(pool, store)
    x = torch.zeros(1, H, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="top-k"):
        mod(x, torch.arange(8, dtype=torch.int32, device=cuda).reshape(1, 8))


def test_block_fused_and_streamed_agree(layer, cuda):
    L, store = layer
    g = torch.Generator(device=cuda)
    g.manual_seed(0)
    gw = (torch.randn(E, H, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    gb = torch.randn(E, generator=g, device=cuda)
    spec, quant = L.spec, {"bits": 4, "group_size": 64, "mode": "affine"}
    whole = MoEBlock(0, H, I, E, K, "olmoe", gw, gb, spec, quant, switch=_full(L, store, cuda))
    pool = ExpertPool(0, None, E, 16, L.spec, device=cuda).build()
    streamed = MoEBlock(0, H, I, E, K, "olmoe", gw, gb, spec, quant,
                        switch=StreamingSwitchGLU(pool, store))
    rng = np.random.default_rng(8)
    for t in range(20):
        x = bf16_tensor(affine.bf16_round(rng.standard_normal((1, H)).astype(np.float32)))
        # the resident block's one-token layer on the three-kernel chain: the same bits as
        # the streamed route -> switch -> combine
        prev = _lib.set_path("chain")
        try:
            assert torch.equal(whole(x), streamed(x)), f"step {t}"
        finally:
            _lib.set_path(prev)
        # on the persistent tensor-core kernel (the default): the parity bar
        assert_close(whole(x).float().cpu().numpy(), streamed(x).float().cpu().numpy())
