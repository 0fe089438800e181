"""Policy parity: every policy reproduces the reference's miss counts on its shipped trace.

Goldens come from the reference's own bigrig_engine/pool.py and policies/ run on
data/traces/qwen3_full.npz (tests/golden/make_goldens.py); the known-answer
cases follow tests/test_pool.py:24-52 of the reference.
"""
import json
import os

import numpy as np
import pytest

from bigrig_b200 import pool
from bigrig_b200.pool import LRU, WindowedLFU, _policy_factory, belady, recommended, simulate

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLD, "pool_golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def trace():
    d = np.load(os.path.join(GOLD, "qwen3_trace_l0-3.npz"))
    return d["idx"].astype(np.int64)


def _stream(idx, li):
    T, k = idx.shape[1:]
    return ([int(idx[li, t, r]) for t in range(T) for r in range(k)],
            [r for _t in range(T) for r in range(k)])


POLICIES = ["lru", "wlfu", "lfuda", "s3fifo", "arc", "gaterank"]


@pytest.mark.parametrize("name", POLICIES)
@pytest.mark.parametrize("C", [8, 16, 32, 64])
def test_miss_counts_match_reference_layer0(golden, trace, name, C):
    E = golden["n_experts"]
    seq, ranks = _stream(trace, 0)
    r = simulate(seq, C, E, _policy_factory(name, C, E), ranks)
    assert [r["misses"], r["hits"]] == golden["sim"][f"{name}:0:{C}"]


@pytest.mark.parametrize("name", ["lfuda", "s3fifo"])
@pytest.mark.parametrize("layer", [1, 2, 3])
def test_miss_counts_match_reference_other_layers(golden, trace, name, layer):
    E = golden["n_experts"]
    seq, ranks = _stream(trace, layer)
    for C in (16, 64):
        r = simulate(seq, C, E, _policy_factory(name, C, E), ranks)
        assert [r["misses"], r["hits"]] == golden["sim"][f"{name}:{layer}:{C}"]


@pytest.mark.parametrize("layer", [0, 1, 2, 3])
def test_belady_matches_reference(golden, trace, layer):
    seq, _ = _stream(trace, layer)
    for C in golden["capacities"]:
        b = belady(seq, C)
        assert [b["misses"], b["hits"]] == golden["belady"][f"{layer}:{C}"]


def test_survey_miss_rates(golden):
    # the headline table: layer 0, E=128, requests in router-rank order
    n = 2271 * 8
    want = {16: {"lru": 0.83427, "lfuda": 0.80036, "belady": 0.51057},
            32: {"lru": 0.60678, "lfuda": 0.52989, "belady": 0.29370},
            64: {"lru": 0.21692, "lfuda": 0.16215, "belady": 0.07816}}
    for C, d in want.items():
        assert round(golden["sim"][f"lru:0:{C}"][0] / n, 5) == d["lru"]
        assert round(golden["sim"][f"lfuda:0:{C}"][0] / n, 5) == d["lfuda"]
        assert round(golden["belady"][f"0:{C}"][0] / n, 5) == d["belady"]


def test_known_answers(golden):
    seq = [1, 2, 3, 1, 2, 3, 1, 2, 3]
    r = simulate(seq, 3, 8, LRU)
    assert r["misses"] == 3 and r["hits"] == 6
    assert simulate(seq, 2, 8, LRU)["misses"] == 9
    assert belady(seq, 2)["misses"] < 9
    assert simulate(seq, 8, 8, LRU)["misses"] == 3
    for C in (1, 2, 3, 8):
        s = simulate(seq, C, 8, LRU)
        assert s["hits"] + s["misses"] == len(seq)
        assert s["misses"] == golden["kat"][f"lru:{C}"]
        assert belady(seq, C)["misses"] == golden["kat"][f"belady:{C}"]


def test_belady_is_a_lower_bound_and_matches(golden):
    for case in golden["random"]:
        s, C = case["seq"], case["capacity"]
        b = belady(s, C)["misses"]
        assert b == case["belady"]
        assert simulate(s, C, 12, LRU)["misses"] == case["lru"] >= b
        assert simulate(s, C, 12, WindowedLFU)["misses"] == case["wlfu"] >= b


def test_resolver_finds_every_policy():
    for name in ["lfuda", "s3fifo", "gaterank", "arc", "lru", "wlfu"]:
        p = _policy_factory(name, 16, 128)(16, 128)
        assert hasattr(p, "victim")
    assert pool.available_policies() == ["arc", "gaterank", "lfuda", "lru", "s3fifo",
                                         "windowed_lfu", "wlfu"]
    # any module following the contract resolves by its dotted path
    p = _policy_factory("bigrig_b200.policies.lfuda", 16, 128)(16, 128)
    assert p.name == "lfuda"
    for bad in ("no_such_policy", "_columns"):
        with pytest.raises(ImportError, match="no policy named"):
            _policy_factory(bad, 16, 128)


def test_recommended_is_lfuda():
    d = recommended(16, 128)
    assert d.name == "lfuda"
    f = recommended()
    assert callable(f) and f(16, 128).name == "lfuda"


def test_select_policy_matches_reference(golden, trace, tmp_path, monkeypatch):
    d = tmp_path / "data" / "traces"
    d.mkdir(parents=True)
    np.savez(d / "sel_full.npz", idx=trace, seq_bounds=np.array([0, trace.shape[1]]))
    monkeypatch.setenv("BIGRIG_HOME", str(tmp_path))
    built = ["lfuda", "s3fifo", "gaterank", "arc"]
    for C in ("16", "32"):
        got = pool.select_policy("sel", int(C), layers=2)
        want = golden["select_policy"][C]
        assert sorted(got["policies"]) == sorted(built)
        # the reference ranked more candidates; among these the winner must be the same
        best = max(built, key=lambda n: want["policies"][n]["gap_pct"])
        assert got["best"] == best
        assert got["lru"] == want["lru"] and got["belady"] == want["belady"]
        for n in built:
            assert got["policies"][n]["miss_rate"] == want["policies"][n]["miss_rate"]
            assert got["policies"][n]["gap_pct"] == want["policies"][n]["gap_pct"]


def _audited(seq, C, E, fac, ranks):
    """Capacity never exceeded, the victim always resident (tests/test_pool.py:56-77)."""
    pol = fac(C, E)
    held, bad = set(), []
    for e, rk in zip(seq, ranks):
        if e in held:
            pol.touch(e, rk)
            continue
        if len(held) >= C:
            v = pol.victim()
            if v not in held:
                bad.append(("victim not resident", v))
                if held:
                    held.pop()
            else:
                held.discard(v)
            if hasattr(pol, "evicted"):
                pol.evicted(v)
        held.add(e)
        pol.admit(e, rk)
        if len(held) > C:
            bad.append(("over capacity", len(held)))
    return bad


@pytest.mark.parametrize("name", ["lfuda", "s3fifo", "gaterank", "arc"])
def test_contract_audit(trace, name):
    seq, ranks = _stream(trace[:, :600], 1)
    assert not _audited(seq, 16, 128, _policy_factory(name, 16, 128), ranks)


def test_audit_has_teeth(trace):
    class Cheater(pool.Policy):
        def victim(self):
            return 999999

    class Hoarder(pool.Policy):
        def victim(self):
            return -1

    seq, ranks = _stream(trace[:, :250], 0)
    assert _audited(seq, 8, 128, lambda c, e: Cheater(c, e), ranks)
    assert _audited(seq, 8, 128, lambda c, e: Hoarder(c, e), ranks)


def test_lfuda_exclude_never_names_protected():
    p = recommended(4, 16)
    for e in range(4):
        p.admit(e, 0)
    assert p.victim(exclude={0, 1, 2}) == 3
    assert p.victim(exclude={0, 1, 2, 3}) == -1
