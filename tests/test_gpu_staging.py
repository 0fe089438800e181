"""Next-layer staging: while a capped layer computes, the next layer's own router names its
likely experts and the non-resident ones are copied from pinned host DRAM into staging
buffers; the next layer admits a staged expert with a device-to-device copy.  Staging may
only change where bytes come from, never an answer: a decode through a capped stack gives
the same bits with and without it, with the same pool traffic, and staged experts are used.
"""
import pytest
import torch

from bigrig_b200 import stream
from bigrig_b200.block import fill_store, make_blocks
from bigrig_b200.fetch import HostExpertStore
from bigrig_b200.formats import bytes_per_expert, make_spec

pytestmark = pytest.mark.gpu

LAYERS, H, I, E, K = 4, 1024, 512, 32, 8


def _decode(cuda, staging, steps=16):
    prev = stream.STAGING
    stream.STAGING = staging
    try:
        blocks = make_blocks(LAYERS, H, I, E, K, "olmoe", 4, 64, "float16", True, seed=3,
                             device=cuda)
        spec = make_spec(H, I, 4, 64, "float16")
        store = HostExpertStore({li: (E, bytes_per_expert(spec)) for li in range(LAYERS)})
        fill_store(store, LAYERS, H, I, E, 4, 64, "float16", seed=4, device=cuda)
        handle = stream.attach(blocks, store, 12, policy="lfuda", warm="auto", device=cuda)
        g = torch.Generator(device=cuda)
        g.manual_seed(9)
        outs = []
        for _ in range(steps):
            h = (torch.randn(1, H, generator=g, device=cuda) * 0.5).bfloat16()
            for blk in blocks:
                h = blk(h, residual=h)
            outs.append(h.clone())
        torch.cuda.synchronize()
        st = handle.stats()
        handle.close()
        return torch.cat(outs), st
    finally:
        stream.STAGING = prev


def test_staging_changes_no_answer(cuda):
    on, st_on = _decode(cuda, True)
    off, st_off = _decode(cuda, False)
    assert torch.equal(on, off)
    assert st_on["hits"] == st_off["hits"] and st_on["misses"] == st_off["misses"]
    assert st_off["stage_issued"] == 0
    assert st_on["stage_issued"] > 0
    assert 0 < st_on["stage_hits"] <= st_on["stage_issued"]
    assert st_on["misses"] > 0
