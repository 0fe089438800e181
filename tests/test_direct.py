"""Experts read straight from safetensors shards (bigrig_engine/direct.py) must land in the
host store byte for byte as the packed blob holds them (the reference's invariant,
direct.py:17-21, and tests/test_direct.py's check against a real blob)."""
import json
import os
import struct

import numpy as np
import pytest

from bigrig_b200 import direct, formats
from bigrig_b200.fetch import HostExpertStore

_TAG = {np.dtype(np.uint32): "U32", np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32"}


def _write_shard(path, tensors):
    """A safetensors file: 8-byte header length, JSON table, then the tensors' bytes."""
    table, blobs, pos = {}, [], 0
    for name, arr in tensors.items():
        raw = np.ascontiguousarray(arr).tobytes()
        table[name] = {"dtype": _TAG[arr.dtype], "shape": list(arr.shape),
                       "data_offsets": [pos, pos + len(raw)]}
        blobs.append(raw)
        pos += len(raw)
    head = json.dumps(table).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(head)))
        f.write(head)
        for b in blobs:
            f.write(b)


def _checkpoint(folder, *, plain=False, bias=False, layers=2, E=6, H=128, I=64,
                infix=".mlp.switch_mlp."):
    """Stacked expert tensors over two shards (layer 0 in one, the rest in the other), plus
    dense tensors the loader must skip; returns {layer: [expert arrays]} and the spec."""
    rng = np.random.default_rng(0)
    spec = formats.make_spec(H, I, 4, 64, "bfloat16", plain=plain, bias=bias)
    per_layer, shards = {}, [{}, {}]
    for li in range(layers):
        experts = [{p: {} for p in spec} for _ in range(E)]
        shard = shards[0 if li == 0 else 1]
        for p, comps in spec.items():
            for c, meta in comps.items():
                dt = np.uint32 if meta["dtype"] == "uint32" else np.uint16
                stacked = rng.integers(0, 2**16, size=[E] + meta["shape"]).astype(dt)
                shard[f"model.layers.{li}{infix}{p}.{c}"] = stacked
                for e in range(E):
                    experts[e][p][c] = stacked[e]
        shard[f"model.layers.{li}.self_attn.q_proj.weight"] = rng.standard_normal((4, 4)).astype(np.float32)
        per_layer[li] = experts
    os.makedirs(folder, exist_ok=True)
    _write_shard(os.path.join(folder, "model-00001-of-00002.safetensors"), shards[0])
    _write_shard(os.path.join(folder, "model-00002-of-00002.safetensors"), shards[1])
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump({"num_experts_per_tok": 2, "quantization": {"bits": 4, "group_size": 64}}, f)
    return per_layer, spec


@pytest.mark.parametrize("plain,bias,infix", [(False, False, ".mlp.switch_mlp."),
                                              (True, True, ".block_sparse_moe.experts."),
                                              (False, True, ".ffn.experts.")])
def test_direct_matches_packed_blob(tmp_path, plain, bias, infix):
    per_layer, spec = _checkpoint(str(tmp_path / "model"), plain=plain, bias=bias, infix=infix)
    man = direct.expert_manifest(str(tmp_path / "model"))
    assert man["direct"] and man["top_k"] == 2
    assert set(man["layers"]) == {"0", "1"}
    for li, info in man["layers"].items():
        assert info["spec"] == spec                       # same order, shapes, byte counts
        assert info["bytes_per_expert"] == formats.bytes_per_expert(spec)
        assert info["quant"] == {"bits": 4, "group_size": 64, "mode": "affine"}
        formats.layout_from_spec(info["spec"], info["quant"])   # a layout the kernels take
    got = HostExpertStore.from_direct(str(tmp_path / "model"), pin=False)
    blob = str(tmp_path / "experts.bin")
    q = {"bits": 4, "group_size": 64, "mode": "affine"}
    bman = formats.write_blob(blob, {li: (spec, q, ex) for li, ex in per_layer.items()})
    want = HostExpertStore.from_blob(blob, bman, pin=False)
    for li in per_layer:
        np.testing.assert_array_equal(got.layers[li].numpy(), want.layers[li].numpy())
    # the per-expert segments read the same bytes as the store holds
    seg = direct.expert_segments(man, 1, 3)
    raw = b"".join(open(p, "rb").read()[o:o + n] for p, o, n in seg)
    assert raw == want.layers[1][3].numpy().tobytes()


def test_direct_refuses_bad_checkpoints(tmp_path):
    folder = str(tmp_path / "m")
    _checkpoint(folder)
    shard = os.path.join(folder, "model-00001-of-00002.safetensors")
    # a tensor whose offsets run past the end of its file
    table, start = direct.read_header(shard)
    name = next(n for n in table if "gate_proj.weight" in n)
    table[name]["data_offsets"][1] += 1 << 20
    head = json.dumps(table).encode()
    body = open(shard, "rb").read()[start:]
    with open(shard, "wb") as f:
        f.write(struct.pack("<Q", len(head)) + head + body)
    with pytest.raises(ValueError, match="past the end"):
        direct.expert_manifest(folder)
    # a layer missing a projection
    folder2 = str(tmp_path / "m2")
    _checkpoint(folder2)
    for shard in (os.path.join(folder2, f) for f in os.listdir(folder2) if f.endswith(".safetensors")):
        table, start = direct.read_header(shard)
        data = open(shard, "rb").read()[start:]
        kept = {n: m for n, m in table.items() if ".1.mlp.switch_mlp.up_proj" not in n}
        head = json.dumps(kept).encode()
        with open(shard, "wb") as f:
            f.write(struct.pack("<Q", len(head)) + head + data)
    with pytest.raises(ValueError, match="has no up_proj"):
        direct.expert_manifest(folder2)
    # experts in a layout that is not built
    folder3 = str(tmp_path / "m3")
    os.makedirs(folder3)
    _write_shard(os.path.join(folder3, "a.safetensors"),
                 {"model.layers.0.mlp.experts.w13.weight": np.zeros((4, 8, 8), np.uint32)})
    with open(os.path.join(folder3, "config.json"), "w") as f:
        json.dump({}, f)
    with pytest.raises(ValueError, match="w13"):
        direct.expert_manifest(folder3)
    with pytest.raises(FileNotFoundError):
        direct.scan(str(tmp_path / "nothing"))


def test_quant_rule():
    spec_q = formats.make_spec(128, 64)
    spec_plain = {"gate_proj": {"weight": {}}}
    cfg = {"quantization": {"bits": 8, "group_size": 32, "model.layers.3.mlp.switch_mlp.gate_proj":
                            {"bits": 4, "group_size": 64}}}
    assert direct.quant_of(cfg, "model.layers.0.mlp.switch_mlp.gate_proj", spec_q) == \
        {"bits": 8, "group_size": 32, "mode": "affine"}
    assert direct.quant_of(cfg, "model.layers.3.mlp.switch_mlp.gate_proj", spec_q)["bits"] == 4
    assert direct.quant_of(cfg, "x", spec_plain) == {}        # no scales: not quantised
    assert direct.quant_of({}, "x", spec_q) == {}
