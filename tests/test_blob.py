"""The packed-blob boundary: formats.write_blob writes the reference's expert-contiguous
blob + manifest (bigrig_engine/stream.py:106-186) and HostExpertStore.from_blob loads it
back into the host store byte for byte.  CPU only."""
import json
import os

import numpy as np
import pytest

from bigrig_b200 import formats
from bigrig_b200.fetch import HostExpertStore
from oracle import affine, moe

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _experts(H, I, E, bits, sd, seed):
    rng = np.random.default_rng(seed)
    spec = formats.make_spec(H, I, bits, 64, sd)
    out = []
    for _ in range(E):
        parts = {}
        for p in moe.PROJ:
            o, i = (H, I) if p == "down_proj" else (I, H)
            w = rng.standard_normal((o, i), dtype=np.float32) * 0.02
            c, s, b = affine.quantize(w, 64, bits, sd)
            parts[p] = {"weight": c, "scales": s, "biases": b}
        out.append(parts)
    return spec, out


def test_blob_roundtrip(tmp_path):
    spec4, ex4 = _experts(128, 64, 3, 4, "float16", 1)
    spec8, ex8 = _experts(64, 128, 2, 8, "bfloat16", 2)
    q4 = {"bits": 4, "group_size": 64, "mode": "affine"}
    q8 = {"bits": 8, "group_size": 64, "mode": "affine"}
    path = str(tmp_path / "m.experts.bin")
    # layer 1 given as packed bytes, layer 0 as arrays: both forms land identically
    packed8 = [formats.pack_expert(e, spec8).tobytes() for e in ex8]
    man = formats.write_blob(path, {1: (spec8, q8, packed8), 0: (spec4, q4, ex4)}, top_k=2)
    assert man["total_bytes"] == os.path.getsize(path)
    assert man == formats.load_manifest(path)
    regions = formats.manifest_regions(man)
    assert sorted(regions) == [(0, 0), (0, 1), (0, 2), (1, 0), (1, 1)]
    # expert-contiguous, in order, no gaps
    ends = [0]
    for key in sorted(regions, key=lambda kv: regions[kv][0]):
        off, n = regions[key]
        assert off == ends[-1]
        ends.append(off + n)
    store = HostExpertStore.from_blob(path, man, pin=False)
    for e in range(3):
        assert np.array_equal(store.layers[0][e].numpy(), formats.pack_expert(ex4[e], spec4))
    for e in range(2):
        assert store.layers[1][e].numpy().tobytes() == packed8[e]
    # the store's bytes unpack to the arrays they came from
    back = formats.unpack_expert(store.layers[0][2].numpy(), spec4)
    assert np.array_equal(back["down_proj"]["scales"], ex4[2]["down_proj"]["scales"])
    # the layout the kernels read follows from the manifest's spec and quant
    L = formats.layout_from_spec(man["layers"]["0"]["spec"], man["layers"]["0"]["quant"])
    assert L.bytes_per_expert == man["layers"]["0"]["bytes_per_expert"]


def test_blob_rejects_wrong_sizes(tmp_path):
    spec, ex = _experts(128, 64, 1, 4, "float16", 3)
    blob = formats.pack_expert(ex[0], spec).tobytes()
    with pytest.raises(ValueError, match="accounts for"):
        formats.write_blob(str(tmp_path / "b.bin"), {0: (spec, None, [blob[:-4]])})
    man = formats.write_blob(str(tmp_path / "c.bin"), {0: (spec, None, [blob])})
    man["layers"]["0"]["bytes_per_expert"] += 4
    with pytest.raises(ValueError, match="region 0:0"):
        HostExpertStore.from_blob(str(tmp_path / "c.bin"), man, pin=False)


def test_manifest_layout_matches_shipped_olmoe(tmp_path):
    """A blob written for the OLMoE shape has the byte layout of the reference's shipped
    OLMoE manifest (tests/golden/manifest_golden.json)."""
    with open(os.path.join(GOLD, "manifest_golden.json")) as f:
        gold = json.load(f)
    g = gold["OLMoE-1B-7B-0125-4bit"]
    spec = formats.make_spec(2048, 1024, 4, 64, "float16")
    assert spec == g["layer0"]["spec"]
    blobs = [bytes(formats.bytes_per_expert(spec))] * 3
    man = formats.write_blob(str(tmp_path / "o.bin"), {0: (spec, g["layer0"]["quant"], blobs)})
    head = dict(list(g["regions_head"].items())[:3])
    assert {k: man["regions"][k] for k in head} == head
    assert man["layers"]["0"]["bytes_per_expert"] == g["layer0"]["bytes_per_expert"]
