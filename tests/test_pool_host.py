"""ExpertPool / ensure bookkeeping against the reference's own pool, replayed step by step.

tests/golden/ensure_golden.npz holds the slot ids the reference's ExpertPool +
StreamingSwitchGLU.ensure (bigrig_engine/stream.py:454-810, 922-978) returned on
a 400-step decode stream and on the expert-sorted spans of a 96-token prompt,
with its final tables and counters.  The pool here runs on a CPU slab for this
test (residency logic only; the compute path has no CPU implementation).
"""
import os

import numpy as np
import pytest
import torch

from bigrig_b200.fetch import HostExpertStore
from bigrig_b200.formats import make_spec
from bigrig_b200.stream import ExpertPool, StreamingSwitchGLU, StreamHandle, _pair_chunks

GOLD = os.path.join(os.path.dirname(__file__), "golden")
SPEC = make_spec(64, 64, 4, 64, "float16")


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(os.path.join(GOLD, "ensure_golden.npz")))


def _store(E):
    st = HostExpertStore({0: (E, sum(c["nbytes"] for p in SPEC.values() for c in p.values()))},
                         pin=False)
    for e in range(E):
        st.layers[0][e].fill_(e % 251)
    return st


def _module(name, C, E=128):
    pool = ExpertPool(0, None, E, C, SPEC, policy=name, device="cpu").build()
    return StreamingSwitchGLU(pool, _store(E))


@pytest.mark.parametrize("name", ["lfuda", "lru", "arc", "s3fifo", "gaterank"])
@pytest.mark.parametrize("C", [8, 12, 40])
def test_decode_replay_matches_reference(golden, name, C):
    mod = _module(name, C)
    toks = golden["decode_tokens"].astype(np.int64)
    slots = np.stack([mod.ensure(toks[t:t + 1]) for t in range(toks.shape[0])]).reshape(toks.shape)
    key = f"{name}:{C}"
    np.testing.assert_array_equal(slots, golden[f"decode_slots:{key}"])
    p = mod._pool
    np.testing.assert_array_equal(np.concatenate([p.g2s, p.s2g]), golden[f"decode_tables:{key}"])
    assert [p.hits, p.misses, p.admits, p.evicts] == golden[f"decode_counts:{key}"].tolist()
    # every resident slot holds exactly the bytes of the expert the table names
    for slot, e in enumerate(p.s2g):
        if e >= 0:
            assert torch.all(p.slab[slot, :p.layout.bytes_per_expert] == e % 251)


@pytest.mark.parametrize("name", ["lfuda", "lru", "arc", "s3fifo", "gaterank"])
@pytest.mark.parametrize("C", [8, 12, 40])
def test_prefill_spans_match_reference(golden, name, C):
    mod = _module(name, C)
    toks = golden["decode_tokens"].astype(np.int64)
    for t in range(toks.shape[0]):
        mod.ensure(toks[t:t + 1])
    pf = golden["prefill_tokens"].astype(np.int64)
    pe = pf.reshape(-1)
    order = np.argsort(pe, kind="stable")
    spe, rank = pe[order], order % pf.shape[1]
    got = np.concatenate([mod.ensure(spe[lo:hi], ranks=rank[lo:hi]).reshape(-1)
                          for lo, hi in _pair_chunks(spe, C)])
    key = f"{name}:{C}"
    np.testing.assert_array_equal(got, golden[f"prefill_slots:{key}"])
    p = mod._pool
    np.testing.assert_array_equal(np.concatenate([p.g2s, p.s2g]), golden[f"prefill_tables:{key}"])
    assert [p.hits, p.misses, p.admits, p.evicts] == golden[f"prefill_counts:{key}"].tolist()


def test_pair_chunks_are_legal():
    rng = np.random.default_rng(3)
    for T, k, E, C in ((69, 8, 128, 11), (5, 8, 64, 8), (300, 4, 128, 16), (1, 2, 8, 2)):
        idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)])
        spe = np.sort(idx.reshape(-1), kind="stable")
        spans = _pair_chunks(spe, C)
        assert spans[0][0] == 0 and spans[-1][1] == spe.size
        for (lo, hi), (lo2, _) in zip(spans, spans[1:]):
            assert hi == lo2
        for lo, hi in spans:
            assert len(np.unique(spe[lo:hi])) <= C
        # an expert never straddles two spans
        owners = {}
        for j, (lo, hi) in enumerate(spans):
            for e in np.unique(spe[lo:hi]):
                assert owners.setdefault(int(e), j) == j


def test_pool_errors():
    with pytest.raises(ValueError, match="capacity must be in"):
        ExpertPool(0, None, 16, 0, SPEC, device="cpu")
    with pytest.raises(ValueError, match="capacity must be in"):
        ExpertPool(0, None, 16, 17, SPEC, device="cpu")
    p = ExpertPool(0, None, 16, 4, SPEC, device="cpu")
    bpe = p.bytes_per_expert
    with pytest.raises(RuntimeError, match="build"):
        p.admit(0, bytes(bpe))
    p.build()
    with pytest.raises(ValueError, match="nothing is written"):
        p.admit(0, bytes(bpe - 1))
    for e in range(4):
        p.touch([e], [0])
        p.admit(e, bytes(bpe))
    with pytest.raises(RuntimeError, match="top-k"):
        p._victim(protect={0, 1, 2, 3})


def test_ensure_rejects_more_misses_than_slots():
    mod = _module("lfuda", 8, E=64)
    with pytest.raises(RuntimeError, match="at least top-k"):
        mod.ensure(np.arange(16).reshape(2, 8))


def test_warm_auto_fills_only_whole_layers():
    E = 16
    st = HostExpertStore({0: (E, sum(c["nbytes"] for p in SPEC.values() for c in p.values())),
                          1: (E, sum(c["nbytes"] for p in SPEC.values() for c in p.values()))},
                         pin=False)
    pools = [ExpertPool(0, None, E, E, SPEC, device="cpu").build(),
             ExpertPool(1, None, E, 4, SPEC, device="cpu").build()]
    mods = [StreamingSwitchGLU(p, st) for p in pools]
    h = StreamHandle(None, pools, mods, st).warm("auto")
    assert pools[0].full and not pools[1].full
    assert [m.refresh() for m in mods] == [True, False]
    assert pools[0].hits == pools[0].misses == 0
    s = h.stats()
    assert s["full_layers"] == 1 and s["sync_free"] == 1
    with pytest.raises(ValueError):
        h.warm("sometimes")


def test_usage_roundtrip(tmp_path):
    mod = _module("lfuda", 8, E=32)
    mod.ensure(np.array([[1, 2, 3, 4, 5, 6, 7, 8]]))
    h = StreamHandle(None, [mod._pool], [mod], mod._fetcher)
    path = str(tmp_path / "usage.json")
    h.save_usage(path)
    h.save_usage(path)
    import json
    d = json.load(open(path))
    assert d["0:1"] == 1      # the earlier count halves to 0 and drops; this run adds 1
