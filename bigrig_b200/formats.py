"""The packed expert format: per-layer spec, byte layout of one expert, and packing.

One expert is one contiguous byte region, its projections in the order the
reference packs them (bigrig_engine/stream.py:106-186, ``PROJECTIONS`` at
stream.py:55 and ``COMPONENTS`` at stream.py:79): gate_proj, up_proj, down_proj,
each as weight (uint32 codes), scales, biases, and an optional affine ``bias``.
The manifest ``spec`` of a layer gives each component's shape, dtype and byte
count; ``bytes_per_expert`` is their sum.  For OLMoE-1B-7B 4-bit that is
3,538,944 bytes (data/blobs/OLMoE-1B-7B-0125-4bit.experts.manifest.json).

A slot of the HBM slab holds exactly these bytes, so admitting an expert is one
copy of its region; the kernels read it in place through ``ExpertLayout``.
"""
from __future__ import annotations

import dataclasses
import json
import os

import numpy as np

PROJECTIONS = ("gate_proj", "up_proj", "down_proj")
MLP_PROJECTIONS = ("fc1", "fc2")          # the plain two-layer expert (stream.py:56)
COMPONENTS = ("weight", "scales", "biases", "bias")
# the activation ids of the layout flags (BIGRIG_ACT_* in include/bigrig_b200.h)
ACTIVATIONS = {"silu": 0, "swiglu": 0, "gpt_oss": 1, "relu2": 2}
FLAG_PLAIN, FLAG_BIAS = 1, 2
_DTYPE_CODE = {"float32": 0, "float16": 1, "bfloat16": 2}
_NP = {"uint32": np.uint32, "float16": np.uint16, "bfloat16": np.uint16, "float32": np.float32,
       "uint8": np.uint8}
_SIZE = {"uint32": 4, "float16": 2, "bfloat16": 2, "float32": 4, "uint8": 1}


def make_spec(hidden: int, inter: int, bits: int = 4, group_size: int = 64,
              scale_dtype: str = "float16", *, plain: bool = False, bias: bool = False,
              bias_dtype: str = "bfloat16", order=None) -> dict:
    """The manifest spec of an expert in MLX affine format (3, 4 or 8 bits): the gated
    gate/up/down expert, or with ``plain`` the fc1/fc2 one; ``bias`` adds each
    projection's affine bias ``[out]`` of ``bias_dtype``; ``order`` lists the components of
    every projection in the order the bytes are packed (the default: weight, scales,
    biases, bias)."""
    if bits not in (3, 4, 8):
        raise ValueError(f"bits must be 3, 4 or 8, got {bits}")
    spec = {}
    for proj in (MLP_PROJECTIONS if plain else PROJECTIONS):
        out_dim, in_dim = (hidden, inter) if proj in ("down_proj", "fc2") else (inter, hidden)
        if in_dim % group_size or (in_dim * bits) % 32:
            raise ValueError(f"{proj}: in={in_dim} is not a multiple of group_size={group_size} "
                             f"or does not fill whole words at {bits} bits")
        words = in_dim * bits // 32
        groups = in_dim // group_size
        spec[proj] = {
            "weight": {"shape": [out_dim, words], "dtype": "uint32", "nbytes": out_dim * words * 4},
            "scales": {"shape": [out_dim, groups], "dtype": scale_dtype, "nbytes": out_dim * groups * 2},
            "biases": {"shape": [out_dim, groups], "dtype": scale_dtype, "nbytes": out_dim * groups * 2},
        }
        if bias:
            spec[proj]["bias"] = {"shape": [out_dim], "dtype": bias_dtype,
                                  "nbytes": out_dim * _SIZE[bias_dtype]}
        if order is not None:
            spec[proj] = {c: spec[proj][c] for c in order if c in spec[proj]}
    return spec


def bytes_per_expert(spec: dict) -> int:
    return sum(c["nbytes"] for p in spec.values() for c in p.values())


def component_offsets(spec: dict) -> dict:
    """{(proj, comp): byte offset inside one expert}, in packing order."""
    out, pos = {}, 0
    for proj in spec:
        for comp, meta in spec[proj].items():
            out[(proj, comp)] = pos
            pos += meta["nbytes"]
    return out


@dataclasses.dataclass(frozen=True)
class Layout:
    """Python view of ``bigrig_expert_layout`` for one layer's experts."""
    hidden: int
    inter: int
    bits: int
    group_size: int
    scale_dtype: str
    bytes_per_expert: int
    slot_stride: int
    weight_off: tuple
    scales_off: tuple
    biases_off: tuple
    source_bits: int = 0        # bits of the stored codes when admission widens them (3), else 0
    source_bytes: int = 0       # one stored expert's bytes when they differ from the slot's
    flags: int = 0              # FLAG_PLAIN | FLAG_BIAS | bias dtype << 2 | activation << 8
    bias_off: tuple = (0, 0, 0)

    @property
    def scale_code(self) -> int:
        return {"float16": 1, "bfloat16": 2}[self.scale_dtype]

    @property
    def plain(self) -> bool:
        return bool(self.flags & FLAG_PLAIN)

    @property
    def has_bias(self) -> bool:
        return bool(self.flags & FLAG_BIAS)

    @property
    def activation(self) -> int:
        return (self.flags >> 8) & 15

    def with_activation(self, name: str | None) -> "Layout":
        """This layout computing ``name`` ("silu"/"swiglu", "gpt_oss" for gated experts,
        "relu2" for plain ones; None: SiLU)."""
        act = ACTIVATIONS.get(name or "silu")
        if act is None:
            raise NotImplementedError(f"activation {name!r}: built are {sorted(ACTIVATIONS)}")
        if (act == 1 and self.plain) or (act == 2 and not self.plain):
            raise NotImplementedError(f"activation {name!r} is not built for the "
                                      f"{'plain fc1/fc2' if self.plain else 'gated'} expert")
        return dataclasses.replace(self, flags=(self.flags & ~(15 << 8)) | (act << 8))


def layout_from_spec(spec: dict, quant: dict | None = None, slot_align: int = 256) -> Layout:
    """The kernel layout of an affine-quantised expert spec: gated (gate/up/down) or plain
    (fc1/fc2), each projection with weight, scales and biases and optionally the affine
    ``bias``, components in any packed order.  Raises NotImplementedError for what is not
    built and ValueError for an inconsistent spec."""
    projs = tuple(spec)
    if projs == PROJECTIONS:
        plain, idx = False, {"gate_proj": 0, "up_proj": 1, "down_proj": 2}
    elif projs == MLP_PROJECTIONS:
        plain, idx = True, {"fc1": 0, "fc2": 2}
    else:
        raise NotImplementedError(f"projections {projs}: built are {PROJECTIONS} (gated) and "
                                  f"{MLP_PROJECTIONS} (plain)")
    for proj in projs:
        for comp in ("weight", "scales", "biases"):
            if comp not in spec[proj]:
                raise NotImplementedError(f"{proj} lacks {comp}: only affine-quantised experts")
        unknown = set(spec[proj]) - set(COMPONENTS)
        if unknown:
            raise ValueError(f"{proj}: unknown components {sorted(unknown)}")
    with_bias = ["bias" in spec[p] for p in projs]
    if any(with_bias) and not all(with_bias):
        raise NotImplementedError("an affine bias on some projections only")
    bias_dtype = spec[projs[0]]["bias"]["dtype"] if with_bias[0] else None
    if bias_dtype is not None and any(spec[p]["bias"]["dtype"] != bias_dtype for p in projs):
        raise NotImplementedError("affine biases of different dtypes")
    if bias_dtype is not None and bias_dtype not in _DTYPE_CODE:
        raise NotImplementedError(f"bias dtype {bias_dtype}")
    q = dict(quant or {"bits": 4, "group_size": 64, "mode": "affine"})
    if q.get("mode", "affine") != "affine":
        raise NotImplementedError(f"quant mode {q.get('mode')!r}: only affine is built")
    bits, gs = int(q["bits"]), int(q["group_size"])
    first, last = projs[0], projs[-1]
    sd = spec[first]["scales"]["dtype"]
    if bits == 3:
        # stored as 3-bit code streams, held in HBM widened to 4-bit codes (lossless: the
        # same q, scales and biases); the slot layout is the 4-bit one
        if plain or bias_dtype is not None:
            raise NotImplementedError("3-bit codes of the gated expert without biases only")
        gw = spec["gate_proj"]["weight"]["shape"]
        inter, hidden = gw[0], gw[1] * 32 // 3
        wide = layout_from_spec(make_spec(hidden, inter, 4, gs, sd),
                                {"bits": 4, "group_size": gs, "mode": "affine"}, slot_align)
        if make_spec(hidden, inter, 3, gs, sd) != spec:
            raise ValueError("a 3-bit spec whose shapes or order are not gate, up, down of "
                             "weight, scales, biases")
        return dataclasses.replace(wide, source_bits=3, source_bytes=bytes_per_expert(spec))
    if bits not in (4, 8):
        raise NotImplementedError(f"{bits}-bit experts: 3-, 4- and 8-bit affine codes are built")
    gw = spec[first]["weight"]["shape"]
    dw = spec[last]["weight"]["shape"]
    inter, hidden = gw[0], gw[1] * 32 // bits
    if dw != [hidden, inter * bits // 32]:
        raise ValueError(f"{last} weight {dw} does not match {first} {gw}")
    if bias_dtype is not None:
        for p in projs:
            out_dim = hidden if p == last else inter
            if spec[p]["bias"]["shape"] != [out_dim]:
                raise ValueError(f"{p}.bias shape {spec[p]['bias']['shape']}, want [{out_dim}]")
    offs = component_offsets(spec)
    bpe = bytes_per_expert(spec)
    stride = (bpe + slot_align - 1) // slot_align * slot_align

    def per_proj(comp):
        out = [0, 0, 0]
        for p, i in idx.items():
            if comp in spec[p]:
                out[i] = offs[(p, comp)]
        return tuple(out)

    flags = (FLAG_PLAIN if plain else 0)
    if bias_dtype is not None:
        flags |= FLAG_BIAS | (_DTYPE_CODE[bias_dtype] << 2)
    return Layout(hidden=hidden, inter=inter, bits=bits, group_size=gs, scale_dtype=sd,
                  bytes_per_expert=bpe, slot_stride=stride, weight_off=per_proj("weight"),
                  scales_off=per_proj("scales"), biases_off=per_proj("biases"), flags=flags,
                  bias_off=per_proj("bias"))


def pack_expert(arrays: dict, spec: dict) -> np.ndarray:
    """{proj: {comp: ndarray}} -> the expert's bytes (uint8) in spec order, length-checked."""
    parts = []
    for proj in spec:
        for comp, meta in spec[proj].items():
            a = np.ascontiguousarray(arrays[proj][comp])
            b = a.view(np.uint8).reshape(-1)
            if b.nbytes != meta["nbytes"]:
                raise ValueError(f"{proj}.{comp}: {b.nbytes} bytes, spec says {meta['nbytes']}")
            parts.append(b)
    return np.concatenate(parts)


def unpack_expert(blob, spec: dict) -> dict:
    """The inverse of pack_expert: {proj: {comp: ndarray}} views of ``blob``."""
    buf = np.frombuffer(blob, dtype=np.uint8) if not isinstance(blob, np.ndarray) else blob
    if buf.nbytes != bytes_per_expert(spec):
        raise ValueError(f"blob of {buf.nbytes} bytes, spec accounts for {bytes_per_expert(spec)}")
    out, pos = {}, 0
    for proj in spec:
        out[proj] = {}
        for comp, meta in spec[proj].items():
            n = meta["nbytes"]
            out[proj][comp] = buf[pos:pos + n].view(_NP[meta["dtype"]]).reshape(meta["shape"])
            pos += n
    return out


# ------------------------------------------------------------------ manifests
def load_manifest(path: str) -> dict:
    """Read a packed-blob manifest (``<blob>.manifest.json``, version >= 4)."""
    p = path if path.endswith(".manifest.json") else path + ".manifest.json"
    if not os.path.exists(p):
        raise FileNotFoundError(f"{p} not found: a blob without its manifest has no byte layout")
    with open(p) as f:
        m = json.load(f)
    for key in ("regions", "layers", "total_bytes"):
        if key not in m:
            raise ValueError(f"{p}: manifest lacks {key!r}")
    return m


def manifest_regions(manifest: dict) -> dict:
    """{(layer, expert): (offset, length)} from a manifest's ``regions``."""
    return {tuple(int(x) for x in k.split(":")): (int(o), int(n))
            for k, (o, n) in manifest["regions"].items()}


def write_blob(path: str, layers: dict, top_k: int | None = None) -> dict:
    """Write experts as one expert-contiguous blob plus ``<path>.manifest.json``; return the
    manifest (the reference's packed-blob format, bigrig_engine/stream.py:106-186).

    ``layers``: {layer: (spec, quant, experts)} where ``experts`` is a sequence whose item e
    is expert e as packed bytes (anything ``np.frombuffer`` takes, or a uint8 array) or as
    {proj: {comp: ndarray}} (packed here with ``pack_expert``).  Layers go in ascending
    order, experts in id order, each expert's bytes in one region; every region is checked
    against the spec's byte count before anything is written for it."""
    manifest = {"version": 4, "layers": {}, "regions": {}}
    pos = 0
    folder = os.path.dirname(os.path.abspath(path))
    os.makedirs(folder, exist_ok=True)
    with open(path, "wb") as out:
        for li in sorted(int(x) for x in layers):
            spec, quant, experts = layers[li]
            want = bytes_per_expert(spec)
            entry = {"n_experts": len(experts), "spec": spec, "bytes_per_expert": want}
            if quant:
                entry["quant"] = dict(quant)
            manifest["layers"][str(li)] = entry
            for e, ex in enumerate(experts):
                data = pack_expert(ex, spec) if isinstance(ex, dict) else (
                    np.asarray(ex, dtype=np.uint8).reshape(-1) if isinstance(ex, np.ndarray)
                    else np.frombuffer(ex, dtype=np.uint8))
                if data.nbytes != want:
                    raise ValueError(f"layer {li} expert {e}: {data.nbytes} bytes, the spec "
                                     f"accounts for {want}")
                out.write(data.tobytes())
                manifest["regions"][f"{li}:{e}"] = [pos, want]
                pos += want
    manifest["total_bytes"] = pos
    if top_k:
        manifest["top_k"] = int(top_k)
    with open(path + ".manifest.json", "w") as f:
        json.dump(manifest, f)
    return manifest
