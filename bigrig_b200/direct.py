"""Experts straight from a model's own safetensors shards into the pinned host store.

Replaces bigrig_engine/direct.py (scan 88-107, quant rule 110-142, expert_manifest
145-240, store 243-246).  The reference points its fetcher INTO the original files and
reads an expert's nine component ranges at every admission.  Here the host store is
filled once at load, so each stacked ``(E, ...)`` component tensor is read from disk in
one pass and its E rows are scattered into the store at that component's offset inside
every expert's region -- one large sequential read per component and layer instead of
E x 9 small ones.  The invariant is the reference's: the bytes of expert e end up exactly
as the packed blob holds them (projection outer, component inner, in ``formats``'
order), so the pool and kernels cannot tell which loader filled the store.
"""
from __future__ import annotations

import glob
import json
import os
import struct
from dataclasses import dataclass

import numpy as np

from .formats import COMPONENTS, MLP_PROJECTIONS, PROJECTIONS

# The module paths under which MoE families keep their stacked expert tensors (a naming
# convention of the checkpoints; the list is the reference's, direct.py:43-45).  Exact
# infixes, not prefixes: shared experts also sit under ``.mlp.``/``.ffn.`` and are dense.
EXPERT_INFIXES = (".mlp.switch_mlp.", ".mlp.experts.", ".feed_forward.experts.",
                  ".ffn.switch_mlp.", ".ffn.experts.", ".mixer.switch_mlp.",
                  ".block_sparse_moe.switch_mlp.", ".block_sparse_moe.experts.")

# safetensors dtype tag -> (manifest dtype name, bytes per element)
DTYPES = {"F64": ("float64", 8), "F32": ("float32", 4), "F16": ("float16", 2),
          "BF16": ("bfloat16", 2), "I64": ("int64", 8), "I32": ("int32", 4),
          "I16": ("int16", 2), "I8": ("int8", 1), "U8": ("uint8", 1),
          "U32": ("uint32", 4), "U16": ("uint16", 2), "BOOL": ("bool_", 1)}

_MAX_HEADER = 1 << 30


@dataclass(frozen=True)
class TensorRef:
    """Where one tensor's bytes sit: file, absolute offset, length, dtype tag, shape."""
    path: str
    offset: int
    nbytes: int
    dtype: str
    shape: tuple


def read_header(path: str) -> tuple:
    """(the shard's tensor table, the file offset where tensor data starts)."""
    with open(path, "rb") as fh:
        head = fh.read(8)
        if len(head) < 8:
            raise ValueError(f"{path}: shorter than a safetensors length prefix")
        (n,) = struct.unpack("<Q", head)
        if n == 0 or n >= _MAX_HEADER:
            raise ValueError(f"{path}: header length {n} is not plausible")
        table = json.loads(fh.read(n))
    if not isinstance(table, dict):
        raise ValueError(f"{path}: the header is not a JSON object")
    return table, 8 + n


def scan(model_dir: str) -> dict:
    """{tensor name: TensorRef} over every ``*.safetensors`` shard of ``model_dir``."""
    root = os.path.expanduser(model_dir)
    shards = sorted(glob.glob(os.path.join(root, "*.safetensors")))
    if not shards:
        raise FileNotFoundError(f"no safetensors shards in {root}")
    refs = {}
    for path in shards:
        table, start = read_header(path)
        size = os.path.getsize(path)
        for name, meta in table.items():
            if name == "__metadata__":
                continue
            lo, hi = (int(v) for v in meta["data_offsets"])
            if hi < lo or start + hi > size:
                raise ValueError(f"{path}: {name} spans bytes {lo}..{hi}, past the end of the "
                                 f"{size}-byte file")
            refs[name] = TensorRef(path, start + lo, hi - lo, meta["dtype"],
                                   tuple(int(d) for d in meta["shape"]))
    return refs


def quant_of(config: dict, module: str, spec: dict) -> dict:
    """A layer's quantisation: {} when its experts carry no ``scales`` (the tensors decide,
    whatever the config says), else the config's per-module entry or its global block."""
    if not any("scales" in comps for comps in spec.values()):
        return {}
    block = config.get("quantization") or config.get("quantization_config") or {}
    if not block:
        return {}
    entry = block.get(module)
    src = entry if isinstance(entry, dict) else block
    return {"bits": int(src.get("bits", 4)), "group_size": int(src.get("group_size", 64)),
            "mode": src.get("mode", "affine")}


def _expert_tensors(refs: dict):
    """{layer: {proj: {comp: name}}}, the infix that matched, and foreign projection names."""
    found, infix_seen, foreign = {}, None, set()
    for name in refs:
        infix = next((i for i in EXPERT_INFIXES if i in name), None)
        if infix is None:
            continue
        head, tail = name.split(infix, 1)
        layer = int(head.rsplit(".", 1)[1])
        proj, comp = tail.rsplit(".", 1)
        if proj not in PROJECTIONS and proj not in MLP_PROJECTIONS:
            foreign.add(proj)
            continue
        if comp in COMPONENTS:
            found.setdefault(layer, {}).setdefault(proj, {})[comp] = name
            infix_seen = infix
    return found, infix_seen, foreign


def expert_manifest(model_dir: str) -> dict:
    """The manifest of a model's experts read in place: the packed-blob manifest's keys
    (``layers`` with ``n_experts``, ``spec``, ``bytes_per_expert``, ``quant``; ``top_k``;
    ``total_bytes``), ``direct: True``, and per layer ``components``: one
    ``[file, offset, bytes per expert]`` per component in packed order, expert e's slice
    starting ``e * bytes per expert`` further in."""
    root = os.path.expanduser(model_dir)
    refs = scan(root)
    with open(os.path.join(root, "config.json")) as fh:
        config = json.load(fh)
    found, infix, foreign = _expert_tensors(refs)
    if not found:
        if foreign:
            raise ValueError(f"{root}: a mixture-of-experts model whose experts use a "
                             f"{'/'.join(sorted(foreign))} layout; built are the gate/up/down "
                             f"and fc1/fc2 layouts")
        raise ValueError(f"{root}: no stacked expert tensors under any of {EXPERT_INFIXES}")
    man = {"version": 4, "direct": True, "model_dir": root, "layers": {}, "total_bytes": 0}
    top_k = config.get("num_experts_per_tok") or config.get("moe_topk")
    if isinstance(top_k, int) and top_k > 0:
        man["top_k"] = top_k
    for layer in sorted(found):
        projs = PROJECTIONS if "gate_proj" in found[layer] else MLP_PROJECTIONS
        spec, parts, n_exp = {}, [], None
        for proj in projs:
            comps = found[layer].get(proj)
            if not comps:
                raise ValueError(f"layer {layer} has no {proj}: the checkpoint is incomplete")
            spec[proj] = {}
            for comp in COMPONENTS:
                if comp not in comps:
                    continue
                ref = refs[comps[comp]]
                if len(ref.shape) < 2:
                    raise ValueError(f"{comps[comp]}: shape {ref.shape} does not lead with E")
                if n_exp is None:
                    n_exp = ref.shape[0]
                elif ref.shape[0] != n_exp:
                    raise ValueError(f"layer {layer}: {comps[comp]} stacks {ref.shape[0]} "
                                     f"experts, a sibling {n_exp}")
                dname, size = DTYPES[ref.dtype]
                per = int(np.prod(ref.shape[1:])) * size
                if per * n_exp != ref.nbytes:
                    raise ValueError(f"{comps[comp]}: {n_exp} x {per} bytes by its shape, "
                                     f"{ref.nbytes} by its offsets")
                spec[proj][comp] = {"shape": list(ref.shape[1:]), "dtype": dname, "nbytes": per}
                parts.append([ref.path, ref.offset, per])
        bpe = sum(p[2] for p in parts)
        man["layers"][str(layer)] = {
            "n_experts": n_exp, "spec": spec, "bytes_per_expert": bpe, "components": parts,
            "quant": quant_of(config, f"model.layers.{layer}{infix}{projs[0]}", spec)}
        man["total_bytes"] += bpe * n_exp
    return man


def expert_segments(manifest: dict, layer: int, e: int) -> list:
    """Expert e's byte ranges ``[file, offset, length]`` in packed order (the reference's
    per-expert ``segments`` entry, direct.py:228-229)."""
    info = manifest["layers"][str(layer)]
    if not 0 <= e < info["n_experts"]:
        raise IndexError(f"expert {e} outside layer {layer}'s {info['n_experts']}")
    return [[path, off + e * per, per] for path, off, per in info["components"]]


def fill_store(store, manifest: dict, chunk_experts: int = 64) -> None:
    """Read every component tensor of every layer once and scatter its per-expert rows into
    ``store.layers[layer][:, column range]`` (the component's place in each expert's packed
    region).  Reads ``chunk_experts`` experts' slices at a time to bound the staging buffer."""
    for key, info in manifest["layers"].items():
        dst = store.layers[int(key)].numpy()
        E, bpe = int(info["n_experts"]), int(info["bytes_per_expert"])
        if dst.shape != (E, bpe):
            raise ValueError(f"layer {key}: the store holds {dst.shape}, the manifest {(E, bpe)}")
        col = 0
        for path, off, per in info["components"]:
            with open(path, "rb") as fh:
                for e0 in range(0, E, chunk_experts):
                    n = min(chunk_experts, E - e0)
                    fh.seek(off + e0 * per)
                    raw = fh.read(n * per)
                    if len(raw) != n * per:
                        raise IOError(f"{path}: short read at {off + e0 * per}")
                    dst[e0:e0 + n, col:col + per] = np.frombuffer(raw, np.uint8).reshape(n, per)
            col += per
        if col != bpe:
            raise ValueError(f"layer {key}: components cover {col} of {bpe} bytes")
