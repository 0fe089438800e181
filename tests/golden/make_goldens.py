"""Generate the golden fixtures of tests/golden/ from the reference's own Python code.

Run where the BigRig tree is readable, with its path in $BIGRIG_REF:

    BIGRIG_REF=<path to the BigRig tree> python tests/golden/make_goldens.py

What it writes (all small, committed; nothing at test time reads the reference):

* ``qwen3_trace_l0-3.npz`` -- layers 0-3 of the reference's shipped routing
  trace data/traces/qwen3_full.npz (idx [4, 2271, 8] as uint8, seq_bounds).
* ``pool_golden.json``     -- miss/hit counts of every policy and of the Belady
  bound from the reference's bigrig_engine/pool.py ``simulate``/``belady`` on
  those layers (requests in router-rank order, pool.py:337-358), the
  ``select_policy`` report, and known-answer sequences of tests/test_pool.py.
* ``ensure_golden.npz``    -- the reference's own ExpertPool + StreamingSwitchGLU
  ``ensure`` bookkeeping (bigrig_engine/stream.py:454-810, 922-978) replayed on a
  decode stream and on expert-sorted prefill spans: the slot ids returned per
  step and the final g2s/s2g tables and counters, per policy and capacity.

stream.py imports mlx at module top (stream.py:41-42) and MLX is not installed
here, so a stand-in ``mlx`` package is placed in sys.modules before the import.
It only has to carry the pool's bookkeeping through: in views mode an admitted
expert's arrays are opaque objects the pool stores and never computes with.
"""
from __future__ import annotations

import json
import os
import sys
import types

import numpy as np

REF = os.environ.get("BIGRIG_REF", "")
HERE = os.path.dirname(os.path.abspath(__file__))
POLICIES = ["lru", "wlfu", "lfuda", "s3fifo", "arc", "lirs", "gaterank", "coact"]
CAPACITIES = [8, 16, 32, 64]
LAYERS = [0, 1, 2, 3]


def _install_mlx_standin() -> None:
    class Opaque:
        def __getitem__(self, _):
            return self

        def __setitem__(self, _k, _v):
            pass

        def view(self, *_a, **_k):
            return self

        def reshape(self, *_a, **_k):
            return self

        def astype(self, *_a, **_k):
            return self

    core = types.ModuleType("mlx.core")
    core.__getattr__ = lambda name: (lambda *a, **k: Opaque())  # noqa: E731
    for dt in ("uint32", "uint8", "float16", "bfloat16", "float32", "int32"):
        setattr(core, dt, dt)
    core.array = lambda *a, **k: Opaque()
    core.from_dlpack = lambda *a, **k: Opaque()
    core.zeros = lambda *a, **k: Opaque()
    core.eval = lambda *a, **k: None
    core.clear_cache = lambda *a, **k: None
    nn = types.ModuleType("mlx.nn")

    class Module:
        def __init__(self, *a, **k):
            pass

    nn.Module = Module
    pkg = types.ModuleType("mlx")
    pkg.core, pkg.nn = core, nn
    sys.modules.update({"mlx": pkg, "mlx.core": core, "mlx.nn": nn})


def trace_fixture() -> np.ndarray:
    d = np.load(os.path.join(REF, "data", "traces", "qwen3_full.npz"))
    idx = d["idx"][LAYERS].astype(np.int64)
    assert idx.min() >= 0 and idx.max() < 256
    np.savez_compressed(os.path.join(HERE, "qwen3_trace_l0-3.npz"), idx=idx.astype(np.uint8),
                        seq_bounds=d["seq_bounds"])
    return idx


def pool_goldens(idx: np.ndarray) -> dict:
    from bigrig_engine import pool
    E = int(idx.max()) + 1
    out = {"n_experts": E, "layers": LAYERS, "capacities": CAPACITIES, "sim": {}, "belady": {}}
    for li, layer in enumerate(LAYERS):
        seq = [int(idx[li, t, r]) for t in range(idx.shape[1]) for r in range(idx.shape[2])]
        ranks = [r for _t in range(idx.shape[1]) for r in range(idx.shape[2])]
        for C in CAPACITIES:
            b = pool.belady(seq, C)
            out["belady"][f"{layer}:{C}"] = [b["misses"], b["hits"]]
            for name in POLICIES:
                fac = pool._policy_factory(name, C, E)
                r = pool.simulate(seq, C, E, fac, ranks)
                out["sim"][f"{name}:{layer}:{C}"] = [r["misses"], r["hits"]]
    # known-answer sequences (tests/test_pool.py:24-52)
    kat = {}
    seq = [1, 2, 3, 1, 2, 3, 1, 2, 3]
    for C in (1, 2, 3, 8):
        kat[f"lru:{C}"] = pool.simulate(seq, C, 8, pool.LRU)["misses"]
        kat[f"belady:{C}"] = pool.belady(seq, C)["misses"]
    rng = np.random.default_rng(0)
    rand = []
    for _trial in range(12):
        s = rng.integers(0, 12, 300).tolist()
        C = int(rng.integers(2, 8))
        rand.append({"seq": s, "capacity": C, "belady": pool.belady(s, C)["misses"],
                     "lru": pool.simulate(s, C, 12, pool.LRU)["misses"],
                     "wlfu": pool.simulate(s, C, 12, pool.WindowedLFU)["misses"]})
    out["kat"] = kat
    out["random"] = rand
    # policy selection on a trace, as select_policy runs it (pool.py:219-249)
    os.environ["BIGRIG_HOME"] = os.path.join(HERE, "_selhome")
    os.makedirs(os.path.join(HERE, "_selhome", "data", "traces"), exist_ok=True)
    tmp = os.path.join(HERE, "_selhome", "data", "traces", "sel_full.npz")
    np.savez(tmp, idx=idx, seq_bounds=np.array([0, idx.shape[1]]))
    try:
        out["select_policy"] = {str(C): pool.select_policy("sel", C, layers=2) for C in (16, 32)}
    finally:
        os.remove(tmp)
        os.removedirs(os.path.join(HERE, "_selhome", "data", "traces"))
        del os.environ["BIGRIG_HOME"]
    return out


class _Fetcher:
    def __init__(self, blobs):
        self.blobs = blobs

    def fetch(self, keys):
        return {k: memoryview(self.blobs[k[1]]) for k in keys}

    def prefetch(self, keys):
        pass

    def drop(self, keys):
        pass

    def warm(self, keys):
        pass


def ensure_goldens(idx: np.ndarray) -> dict:
    from bigrig_engine import stream
    E = int(idx.max()) + 1
    H = I = 64
    spec = {}
    for p in stream.PROJECTIONS:
        o, i = (H, I) if p == "down_proj" else (I, H)
        spec[p] = {"weight": {"shape": [o, i // 8], "dtype": "uint32", "nbytes": o * i // 2},
                   "scales": {"shape": [o, i // 64], "dtype": "float16", "nbytes": o * i // 32},
                   "biases": {"shape": [o, i // 64], "dtype": "float16", "nbytes": o * i // 32}}
    bpe = sum(c["nbytes"] for pr in spec.values() for c in pr.values())
    blobs = {e: bytes([e % 251]) * bpe for e in range(E)}

    class _SG:
        def __init__(self):
            for p in stream.PROJECTIONS:
                setattr(self, p, {c: None for c in spec[p]})

    decode = idx[1, :400]                       # layer 1, 400 decode steps of one token
    prefill = idx[2, :96]                       # layer 2, one 96-token prompt
    out = {"decode_tokens": decode.astype(np.int16), "prefill_tokens": prefill.astype(np.int16)}
    for name in ["lfuda", "lru", "arc", "s3fifo", "lirs", "gaterank", "coact"]:
        for C in (8, 12, 40):
            pool = stream.ExpertPool(0, _SG(), E, C, spec, policy=name, views=True).build()
            mod = stream.StreamingSwitchGLU(pool, _Fetcher(blobs), None, True,
                                            {"group_size": 64, "bits": 4, "mode": "affine"})
            slots = np.stack([mod.ensure(decode[t:t + 1]) for t in range(decode.shape[0])])
            key = f"{name}:{C}"
            out[f"decode_slots:{key}"] = slots.reshape(decode.shape).astype(np.int16)
            out[f"decode_tables:{key}"] = np.concatenate([pool.g2s, pool.s2g]).astype(np.int16)
            out[f"decode_counts:{key}"] = np.array([pool.hits, pool.misses, pool.admits,
                                                    pool.evicts], dtype=np.int64)
            # expert-sorted prefill spans of <= C distinct experts, with ranks
            # (stream.py:1521-1561, _pair_chunks stream.py:1098-1126)
            pe = prefill.reshape(-1)
            order = np.argsort(pe, kind="stable")
            spe = pe[order]
            rank = order % prefill.shape[1]
            sl = []
            for lo, hi in stream.StreamingSwitchGLU._pair_chunks(spe, C):
                sl.append(mod.ensure(spe[lo:hi], ranks=rank[lo:hi]).reshape(-1))
            out[f"prefill_slots:{key}"] = np.concatenate(sl).astype(np.int16)
            out[f"prefill_tables:{key}"] = np.concatenate([pool.g2s, pool.s2g]).astype(np.int16)
            out[f"prefill_counts:{key}"] = np.array([pool.hits, pool.misses, pool.admits,
                                                     pool.evicts], dtype=np.int64)
    return out


def manifest_fixture() -> dict:
    """Layer 0 of each shipped packed-blob manifest plus its first regions and totals."""
    out = {}
    for name in ("OLMoE-1B-7B-0125-4bit", "Qwen3-30B-A3B-3bit"):
        with open(os.path.join(REF, "data", "blobs", f"{name}.experts.manifest.json")) as f:
            m = json.load(f)
        regions = dict(list(m["regions"].items())[:4])
        out[name] = {"layer0": m["layers"]["0"], "n_layers": len(m["layers"]),
                     "regions_head": regions, "total_bytes": m["total_bytes"],
                     "top_k": m.get("top_k"), "version": m.get("version")}
    return out


def main() -> None:
    if not REF or not os.path.isdir(REF):
        raise SystemExit("set BIGRIG_REF to the BigRig tree (the reference's source)")
    sys.path.insert(0, REF)
    with open(os.path.join(HERE, "manifest_golden.json"), "w") as f:
        json.dump(manifest_fixture(), f, indent=1)
    _install_mlx_standin()
    idx = trace_fixture()
    with open(os.path.join(HERE, "pool_golden.json"), "w") as f:
        json.dump(pool_goldens(idx), f)
    np.savez_compressed(os.path.join(HERE, "ensure_golden.npz"), **ensure_goldens(idx))
    print("wrote", sorted(x for x in os.listdir(HERE) if not x.endswith(".py")))


if __name__ == "__main__":
    main()
