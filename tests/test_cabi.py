"""The C-ABI library: it loads without a GPU, exports every symbol include/*.h declares,
and its host-only entry points answer (no device work is issued here)."""
import ctypes
import glob
import os
import re

import pytest

from bigrig_b200 import _lib, formats, ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names |= set(re.findall(r"BIGRIG_API\s+[\w\s\*]+?\b(bigrig_\w+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared()
    assert declared, "no declarations found"
    assert declared == set(_lib.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.bigrig_version().decode().startswith("bigrig_b200")


def test_layout_checks():
    lib = _lib.load()
    L = formats.layout_from_spec(formats.make_spec(2048, 1024, 4, 64, "float16"))
    c = ops.c_layout(L)
    assert lib.bigrig_check_layout(ctypes.byref(c)) == 0
    bad = _lib.ExpertLayout.from_buffer_copy(c)
    bad.bits = 3
    assert lib.bigrig_check_layout(ctypes.byref(bad)) == _lib.ERR_UNSUPPORTED
    bad = _lib.ExpertLayout.from_buffer_copy(c)
    bad.slot_stride = c.bytes_per_expert - 16
    assert lib.bigrig_check_layout(ctypes.byref(bad)) == _lib.ERR_INVALID
    assert "slot_stride" in _lib.last_error()
    bad = _lib.ExpertLayout.from_buffer_copy(c)
    bad.weight_off[2] = c.bytes_per_expert
    assert lib.bigrig_check_layout(ctypes.byref(bad)) == _lib.ERR_INVALID
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ERR_UNSUPPORTED)


def test_workspace_size_grows_with_tokens():
    L = formats.layout_from_spec(formats.make_spec(2048, 1024, 4, 64, "float16"))
    a = ops.workspace_bytes(1, 8, 64, L)
    b = ops.workspace_bytes(128, 8, 64, L)
    assert 0 < a < b
    assert a % 256 == 0


def test_argument_errors_need_no_device():
    lib = _lib.load()
    # invalid top-k is rejected before any device work
    rc = lib.bigrig_router_topk(None, _lib.F32, 4, 64, 0, 0, 0, None, None, None)
    assert rc == _lib.ERR_INVALID
    rc = lib.bigrig_router_topk(None, _lib.F32, 4, 300, 8, 0, 0, None, None, None)
    assert rc == _lib.ERR_UNSUPPORTED
    rc = lib.bigrig_combine(None, None, 1, 8, 7, None, None)
    assert rc == _lib.ERR_INVALID


def test_compute_refuses_cpu_tensors():
    import torch
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        ops.router_logits(torch.zeros(1, 64, dtype=torch.bfloat16),
                          torch.zeros(8, 64, dtype=torch.bfloat16))


def test_peer_group_checks_need_no_device():
    lib = _lib.load()
    assert ctypes.sizeof(_lib.PeerGroup) == 24 + 8 * _lib.PEER_MAX_RANKS
    n1 = lib.bigrig_peer_buffer_bytes(2, 1, 2048, 8)
    n2 = lib.bigrig_peer_buffer_bytes(4, 1, 2048, 8)
    # gathered rows grow with the group, the pair outputs do not
    assert n2 - n1 == 2 * 2048 * 2 and n1 % 256 == 0
    assert lib.bigrig_peer_buffer_bytes(9, 1, 2048, 8) == 0       # more ranks than supported
    L = formats.layout_from_spec(formats.make_spec(2048, 1024, 4, 64, "float16"))
    c = ops.c_layout(L)
    g = _lib.PeerGroup(world=2, rank=0, tokens=1, hidden=2048, top_k=8)
    # a group whose peer buffer is missing is refused before any launch
    g.base[0] = 1 << 20
    rc = lib.bigrig_peer_layer(ctypes.byref(g), None, None, None, 64, 0, 0, 0, 32, None, None,
                               ctypes.byref(c), None, None, None, 0, None)
    assert rc == _lib.ERR_INVALID and "rank 1" in _lib.last_error()
    g.base[1] = 2 << 20
    rc = lib.bigrig_peer_layer(ctypes.byref(g), None, None, None, 64, 0, 0, 48, 32, None, None,
                               ctypes.byref(c), None, None, None, 0, None)
    assert rc == _lib.ERR_INVALID and "outside" in _lib.last_error()
    ws = lib.bigrig_peer_workspace_bytes(ctypes.byref(g), 64, 32, ctypes.byref(c))
    assert ws > ops.workspace_bytes(2, 8, 32, L)
