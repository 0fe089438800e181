"""3-bit experts on the GPU: stored and copied as 3-bit code streams, widened into 4-bit
slots at admission (bigrig_widen_expert), then served by the unchanged expert kernels.

The widened slot must hold exactly the 4-bit packing of the same codes with the same
scales and biases (bit for bit), and the layer over a capped pool of 3-bit experts must
meet the expert parity bar against the restatement dequantising the 3-bit codes
directly, on the GEMV chain, the tcgen05 GEMM and the persistent one-token kernel.
Shapes follow the shipped Qwen3-30B-A3B-3bit manifest's layout at a smaller size."""
import ctypes

import numpy as np
import pytest
import torch

from bigrig_b200 import _lib, formats, ops
from bigrig_b200.fetch import HostExpertStore
from bigrig_b200.stream import ExpertPool, StreamingSwitchGLU
from oracle import affine, moe, router
from tests._experts import assert_close, bf16_tensor, random_routing, to_f32

pytestmark = pytest.mark.gpu

H, I, E, SD = 1024, 512, 16, "bfloat16"


@pytest.fixture(scope="module")
def experts3():
    rng = np.random.default_rng(33)
    spec3 = formats.make_spec(H, I, 3, 64, SD)
    q, blobs = {}, []
    for e in range(E):
        parts, qe = {}, {}
        for p in moe.PROJ:
            o, i = (H, I) if p == "down_proj" else (I, H)
            w = rng.standard_normal((o, i), dtype=np.float32) * 0.02
            c, s, b = affine.quantize(w, 64, 3, SD)
            qe[p] = (c, s, b)
            parts[p] = {"weight": c, "scales": s, "biases": b}
        q[e] = qe
        blobs.append(formats.pack_expert(parts, spec3))
    return spec3, q, blobs


def _wide_bytes(qe):
    spec4 = formats.make_spec(H, I, 4, 64, SD)
    parts = {p: {"weight": affine.pack_codes(affine.unpack_codes(qe[p][0], 3), 4),
                 "scales": qe[p][1], "biases": qe[p][2]} for p in moe.PROJ}
    return formats.pack_expert(parts, spec4)


def test_widen_is_the_4bit_packing_of_the_same_codes(cuda, experts3):
    spec3, q, blobs = experts3
    L = formats.layout_from_spec(spec3, {"bits": 3, "group_size": 64, "mode": "affine"})
    assert L.bits == 4 and L.source_bits == 3 and L.source_bytes == len(blobs[0])
    src = torch.from_numpy(blobs[5]).to(cuda)
    dst = torch.zeros(L.slot_stride, dtype=torch.uint8, device=cuda)
    rc = _lib.load().bigrig_widen_expert(ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(dst.data_ptr()),
                                         ctypes.byref(ops.c_layout(L)), 3,
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dst[:L.bytes_per_expert].cpu().numpy(), _wide_bytes(q[5]))
    # and the dequantised weights of the widened slot are the 3-bit expert's
    for p, proj in enumerate(moe.PROJ):
        rows, cols = (H, I) if p == 2 else (I, H)
        out = torch.empty(rows, cols, dtype=torch.bfloat16, device=cuda)
        _lib.check(_lib.load().bigrig_dequant(ctypes.c_void_p(dst.data_ptr()),
                                              ctypes.byref(ops.c_layout(L)), 0, p,
                                              ctypes.c_void_p(out.data_ptr()), None), "dequant")
        torch.cuda.synchronize()
        want = affine.dequantize(*q[5][proj], 64, 3, SD)
        np.testing.assert_array_equal(out.view(torch.int16).cpu().numpy().view(np.uint16), want)


@pytest.mark.parametrize("path,T", [("gemv", 3), ("gemm", 48), ("auto", 1)])
def test_capped_3bit_pool_meets_the_bar(cuda, experts3, path, T):
    spec3, q, blobs = experts3
    quant = {"bits": 3, "group_size": 64, "mode": "affine"}
    store = HostExpertStore({0: (E, len(blobs[0]))}, pin=True)
    for e in range(E):
        store.put(0, e, blobs[e])
    pool = ExpertPool(0, None, E, 8, spec3, quant=quant, device=cuda).build()
    mod = StreamingSwitchGLU(pool, store)
    rng = np.random.default_rng(T)
    wround, inter = (None, "h_bf16") if path != "gemm" else ("bf16", "h_bf16")
    prev = _lib.set_path("gemm" if path == "gemm" else "gemv" if path == "gemv" else "auto")
    try:
        for step in range(3):
            x = affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
            idx = random_routing(T, 2 if T > 1 else 4, E, rng)
            if len(np.unique(idx)) > 8:
                idx = idx % 8
            if T == 1:
                # one decode token through the whole block on the persistent kernel
                lg = rng.standard_normal((1, E)).astype(np.float32)
                widx, wsc = router.topk(lg, 4)
                mod.ensure(widx)
                pool.ready()
                out = ops.moe_layer_routed(bf16_tensor(x), torch.from_numpy(widx.astype(np.int32)).to(cuda),
                                           torch.from_numpy(wsc.astype(np.float32)).to(cuda), pool.slab,
                                           pool.layout, E, g2s=pool.g2s_device())
                torch.cuda.synchronize()
                ref = moe.combine(moe.switch_glu(x, widx, lambda e: moe.expert_weights_f32(q[e], 64, 3, SD),
                                                 "h_bf16"), wsc)
                assert_close(to_f32(out), ref)
                continue
            y = mod(bf16_tensor(x), torch.from_numpy(idx).to(cuda))
            torch.cuda.synchronize()
            ref = moe.switch_glu(x, idx, lambda e: moe.expert_weights_f32(q[e], 64, 3, SD, wround), inter)
            assert_close(to_f32(y), ref)
    finally:
        _lib.set_path(prev)
    # every resident slot holds the widened bytes of the expert the tables name
    torch.cuda.synchronize()
    for slot, e in enumerate(pool.s2g):
        if e >= 0:
            np.testing.assert_array_equal(pool.slab[slot, :pool.layout.bytes_per_expert].cpu().numpy(),
                                          _wide_bytes(q[int(e)]))
