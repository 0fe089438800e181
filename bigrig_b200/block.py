"""The MoE block around the expert layer: router, SwitchGLU call, weighted combine.

The reference delegates this block to mlx_lm (not in its tree): the gate
produces logits, top-k selects experts with a family-specific softmax order
(bigrig_engine/adapter.py:74-92), the streamed SwitchGLU returns per-(token, k)
outputs and the block sums them weighted by the router scores
(bigrig_engine/stream.py:1523-1525).  Here each step is an sm_100a kernel:
``router_logits`` -> ``router_topk`` -> the layer's ``switch`` -> ``combine``,
or, for a layer whose pool holds every expert, the fused ``moe_forward``.

Also here: quantising synthetic fp32 weights to the MLX affine format on the GPU
(fixtures and benchmarks only; the rule is the one documented for MLX: per group
of 64, scale = (max - min) / (2^bits - 1), bias = min, q = round((w - bias) / scale)).
"""
from __future__ import annotations

import dataclasses

import torch

from . import ops
from .formats import PROJECTIONS, make_spec

FAMILIES = {
    # name: (mode, norm_topk)
    "olmoe": ("softmax_topk", False),
    "qwen3": ("softmax_topk", True),
    "mixtral": ("topk_softmax", False),
    "gpt_oss": ("topk_softmax", False),
}


def quantize_affine(w: torch.Tensor, group_size: int = 64, bits: int = 4,
                    scale_dtype: torch.dtype = torch.float16):
    """fp32 ``w[out, in]`` (any device) -> (uint32 codes [out, in*bits/32] as int32 storage,
    scales [out, in/g], biases [out, in/g]) in ``scale_dtype``."""
    out_dim, in_dim = w.shape
    g = w.float().reshape(out_dim, in_dim // group_size, group_size)
    wmax = g.amax(dim=-1)
    wmin = g.amin(dim=-1)
    n_bins = (1 << bits) - 1
    scale = torch.clamp((wmax - wmin) / float(n_bins), min=1e-7)
    s = scale.to(scale_dtype)
    b = wmin.to(scale_dtype)
    q = torch.clamp(torch.round((g - b.float()[..., None]) / s.float()[..., None]), 0, n_bins)
    q = q.to(torch.int64).reshape(out_dim, in_dim // (32 // bits), 32 // bits)
    shifts = torch.arange(32 // bits, device=w.device, dtype=torch.int64) * bits
    words = (q << shifts).sum(dim=-1)            # < 2^32, exact in int64
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)
    return words, s, b


def pack_expert_tensors(parts: dict) -> torch.Tensor:
    """{proj: (codes int32, scales, biases)} -> one expert's bytes (uint8) in packed order."""
    chunks = []
    for proj in PROJECTIONS:
        for t in parts[proj]:
            chunks.append(t.contiguous().view(torch.uint8).reshape(-1))
    return torch.cat(chunks)


def random_expert_bytes(hidden: int, inter: int, bits: int, group_size: int,
                        scale_dtype: torch.dtype, generator: torch.Generator, device,
                        std: float = 0.02) -> torch.Tensor:
    """One synthetic expert: N(0, std) weights quantised to the affine format, packed."""
    parts = {}
    for proj in PROJECTIONS:
        out_dim, in_dim = (hidden, inter) if proj == "down_proj" else (inter, hidden)
        w = torch.randn(out_dim, in_dim, generator=generator, device=device) * std
        parts[proj] = quantize_affine(w, group_size, bits, scale_dtype)
    return pack_expert_tensors(parts)


@dataclasses.dataclass
class MoEBlock:
    """One MoE layer: router weights plus a SwitchGLU-style ``switch`` (see stream.py)."""
    layer: int
    hidden: int
    inter: int
    n_experts: int
    top_k: int
    family: str
    gate_w: torch.Tensor           # bf16 [E, H]
    gate_b: torch.Tensor | None    # fp32 [E]
    spec: dict
    quant: dict
    switch: object = None

    @property
    def mode(self) -> tuple:
        return FAMILIES[self.family]

    def route(self, x: torch.Tensor):
        logits = ops.router_logits(x, self.gate_w, self.gate_b)
        mode, norm = self.mode
        return ops.router_topk(logits, self.top_k, mode, norm)

    def __call__(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        """x bf16 [T, H] -> combined expert output bf16 [T, H] (+ ``residual`` when given)."""
        mode, norm = self.mode
        sw = self.switch
        pool = getattr(sw, "_pool", None)
        if pool is not None and getattr(sw, "_sync_free", False):
            pool.ready()
            out, _, _ = ops.moe_layer(x, self.gate_w, self.gate_b, self.top_k, pool.slab,
                                      pool.layout, self.n_experts, mode, norm,
                                      g2s=pool.g2s_device(), residual=residual,
                                      workspace=sw.workspace)
            pool.mark_read()
            return out
        if (pool is not None and x.shape[0] == 1 and hasattr(sw, "decode_layer")
                and not getattr(sw, "bypass", False)):
            # one decode token over a capped pool: route, make resident, then the whole
            # layer in one library call
            return sw.decode_layer(x, self.gate_w, self.gate_b, self.top_k, mode, norm,
                                   residual=residual)
        idx, scores = self.route(x)
        y = sw(x, idx)
        return ops.combine(y, scores, residual=residual)


def make_blocks(n_layers: int, hidden: int, inter: int, n_experts: int, top_k: int, family: str,
                bits: int = 4, group_size: int = 64, scale_dtype: str = "float16",
                router_bias: bool = True, seed: int = 0, device="cuda") -> list:
    """Router weights N(0, 0.02) bf16 and per-expert bias N(0, 1) for each layer."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    spec = make_spec(hidden, inter, bits, group_size, scale_dtype)
    quant = {"bits": bits, "group_size": group_size, "mode": "affine"}
    blocks = []
    for li in range(n_layers):
        gw = (torch.randn(n_experts, hidden, generator=g, device=device) * 0.02).to(torch.bfloat16)
        gb = torch.randn(n_experts, generator=g, device=device) if router_bias else None
        blocks.append(MoEBlock(li, hidden, inter, n_experts, top_k, family, gw, gb, spec, quant))
    return blocks


def fill_store(store, n_layers: int, hidden: int, inter: int, n_experts: int, bits: int = 4,
               group_size: int = 64, scale_dtype: str = "float16", seed: int = 1,
               device="cuda", experts=None) -> None:
    """Quantise synthetic experts on the GPU and write them into a HostExpertStore.

    Expert e of layer l is drawn from its own generator (seeded from seed, l, e), so
    a rank holding only a block of experts (``experts``: the global ids to fill, in
    store order) gets exactly the bytes a single GPU holding all of them would."""
    sd = {"float16": torch.float16, "bfloat16": torch.bfloat16}[scale_dtype]
    ids = list(range(n_experts)) if experts is None else list(experts)
    g = torch.Generator(device=device)
    for li in range(n_layers):
        for slot, e in enumerate(ids):
            g.manual_seed(seed * 1_000_003 + li * 10_007 + e)
            b = random_expert_bytes(hidden, inter, bits, group_size, sd, g, device)
            store.layers[li][slot].copy_(b)


class EPMoEBlock:
    """An expert-parallel MoE layer: the replicated router, then ``ep.dispatch_combine``
    to the ranks owning the routed experts, whose ``switch`` (a StreamingSwitchGLU over
    this rank's experts) computes the pairs it receives."""

    def __init__(self, block: MoEBlock, ep, switch, padded: bool):
        self.block, self.ep, self.switch, self.padded = block, ep, switch, padded

    def __call__(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        idx, scores = self.block.route(x)
        sw = self.switch

        def expert_fn(rows, ids):
            return sw(rows.contiguous(), ids.reshape(-1, 1).contiguous()).reshape(rows.shape)

        return self.ep.dispatch_combine(
            x, idx, scores, expert_fn, padded=self.padded,
            combine_fn=lambda y, sc: ops.combine(y.contiguous(), sc, residual=residual))


class EPPeerBlock:
    """An expert-parallel MoE layer whose exchanges are stores into the other ranks' peer
    buffers (``ops.peer_layer``): calls with the group's token count take that path,
    others (a prompt) the NCCL all-to-all block ``fallback``.  The rank's pool must hold
    all of its experts (the layer never reads routing back to the host)."""

    def __init__(self, block: MoEBlock, peers, switch, first: int, n_local: int, fallback=None):
        self.block, self.peers, self.switch = block, peers, switch
        self.first, self.n_local, self.fallback = first, n_local, fallback
        if not switch._pool.full:
            raise ValueError("the peer-memory layer needs every local expert resident")

    @property
    def padded(self) -> bool:
        """The fallback block's exchange mode (a prompt's exact all-to-all, or padded)."""
        return self.fallback.padded

    @padded.setter
    def padded(self, v: bool) -> None:
        self.fallback.padded = v

    def __call__(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        if x.shape[0] != self.peers.tokens:
            return self.fallback(x, residual=residual)
        pool = self.switch._pool
        mode, norm = self.block.mode
        pool.ready()
        out = ops.peer_layer(self.peers, x, self.block.gate_w, self.block.gate_b,
                             self.block.n_experts, self.first, self.n_local, pool.slab,
                             pool.layout, mode, norm, g2s=pool.g2s_device(), residual=residual,
                             workspace=self.switch.workspace)
        pool.mark_read()
        return out
