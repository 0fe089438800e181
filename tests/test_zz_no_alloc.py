"""The allocation-free entry point against the workspace one.

bigrig_switch_glu_noalloc serves callers that cannot allocate device memory when they
call (a process whose device memory another allocator carved up at start-up, or a
latency-critical loop where cudaMalloc's device synchronisation is not allowed): its
scratch is a fixed device array inside the library.  It must give the same experts'
outputs as bigrig_switch_glu on the same inputs, call after call, since every call
reuses the array the previous one left behind.  This file is collected last so that
a run stopping at its first failure has already run everything else.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import affine
from bigrig_b200 import _lib, ops
from tests._experts import Layer, assert_close, bf16_tensor, random_routing, to_f32

pytestmark = pytest.mark.gpu


def test_noalloc_matches_workspace_entry_on_consecutive_calls(cuda):
    rng = np.random.default_rng(77)
    H, I, E, k = 1024, 512, 16, 4
    L = Layer(H, I, E, 4, "float16", seed=77, slot_order=rng.permutation(E))
    lib = _lib.load()
    for T in (3, 1):                       # two calls in a row, different shapes
        x = bf16_tensor(affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32)))
        idx = torch.from_numpy(random_routing(T, k, E, rng)).to(cuda)
        want = ops.switch_glu(x, idx, L.slab, L.layout, E, g2s=L.g2s)
        got = torch.empty_like(want)
        rc = lib.bigrig_switch_glu_noalloc(
            ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(idx.data_ptr()), T, k, E,
            ctypes.c_void_p(L.g2s.data_ptr()), ctypes.c_void_p(L.slab.data_ptr()),
            ctypes.byref(ops.c_layout(L.layout)), ctypes.c_void_p(got.data_ptr()),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert_close(to_f32(got), to_f32(want))


def test_noalloc_takes_the_grouped_gemm_inside_its_scratch(cuda):
    """256 routed pairs: beyond the GEMV chain's 32, so the tcgen05 grouped GEMM runs on
    token rows carved from the static array; two calls in a row."""
    rng = np.random.default_rng(78)
    H, I, E, k, T = 1024, 512, 16, 4, 64
    L = Layer(H, I, E, 4, "float16", seed=78, slot_order=rng.permutation(E))
    assert ops.workspace_bytes(T, k, E, L.layout) <= _lib.NOALLOC_SCRATCH_BYTES
    prev = _lib.set_path("gemm")
    try:
        for _ in range(2):
            x = bf16_tensor(affine.bf16_round(rng.standard_normal((T, H)).astype(np.float32)))
            idx = torch.from_numpy(random_routing(T, k, E, rng)).to(cuda)
            n0 = _lib.launch_counts()["gemm_gate_up"]
            got = ops.switch_glu_noalloc(x, idx, L.slab, L.layout, E, g2s=L.g2s)
            assert _lib.launch_counts()["gemm_gate_up"] == n0 + 1
            want = ops.switch_glu(x, idx, L.slab, L.layout, E, g2s=L.g2s)
            torch.cuda.synchronize()
            assert_close(to_f32(got), to_f32(want))
    finally:
        _lib.set_path(prev)


def test_noalloc_rejects_calls_beyond_its_scratch(cuda):
    H, I, E, k = 1024, 512, 16, 4
    L = Layer(H, I, E, 4, "float16", seed=1)
    T = 2048                               # needs more than the 4 MiB array
    assert ops.workspace_bytes(T, k, E, L.layout) > _lib.NOALLOC_SCRATCH_BYTES
    x = torch.zeros(T, H, dtype=torch.bfloat16, device=cuda)
    idx = torch.zeros(T, k, dtype=torch.int32, device=cuda)
    with pytest.raises(ValueError, match="static array"):
        ops.switch_glu_noalloc(x, idx, L.slab, L.layout, E)
