"""A decoder-only MoE transformer around the expert path: the full decode loop.

The reference runs its MoE models through mlx_lm (attention, KV cache, embeddings, LM
head) and swaps each MoE block's SwitchGLU for the streamed one (bigrig_engine/
stream.py:1842-1958); prefill is layer-major (bigrig_engine/layered.py:85-131), decode
runs one token through every layer (stream.py:1420-1459).  Here the same loop is a thin
torch shell: attention, RoPE, the KV cache and the LM head are bf16 cuBLAS/SDPA calls
(outside the hot path), and every MoE layer is a ``block.MoEBlock`` whose experts live
in this library's pools -- capped pools refilled from pinned host DRAM, or resident.
Weights are random (N(0, 0.02)); norms have unit weight.

Prefill visits the layers in order with the whole prompt at each (the layer-major
schedule: each layer's experts are made resident once for all prompt tokens), filling
the KV cache; decode appends one position per step and picks the next token greedily
on the device.
"""
from __future__ import annotations

import dataclasses

import torch
import torch.nn.functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

# Attention kernels that need no per-shape plan: the cuDNN backend builds an execution plan
# for every new key length (~3 ms of host time per call), i.e. at every decode step.
_SDPA_BACKENDS = [SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]


@dataclasses.dataclass
class AttnConfig:
    """Attention and vocabulary shape of a model family."""
    vocab: int
    heads: int
    kv_heads: int
    head_dim: int = 128
    rope_theta: float = 10000.0
    qk_norm: bool = False
    eps: float = 1e-6


# The attention shapes of the named model families (random init).
FAMILY_ATTN = {
    "olmoe": AttnConfig(vocab=50304, heads=16, kv_heads=16, qk_norm=True),
    "qwen3": AttnConfig(vocab=151936, heads=32, kv_heads=4, qk_norm=True, rope_theta=1e6),
    "mixtral": AttnConfig(vocab=32000, heads=32, kv_heads=8, rope_theta=1e6),
}


class Decoder:
    """Embedding, ``len(blocks)`` decoder layers (attention + the MoE block) and the LM head.

    ``blocks``: the MoE blocks, one per layer, already attached to their pools
    (``stream.attach``) or fused resident layers.  ``max_len``: KV-cache positions."""

    def __init__(self, blocks, attn: AttnConfig, max_len: int, device, seed: int = 0):
        self.blocks = list(blocks)
        self.cfg = attn
        self.device = torch.device(device)
        self.max_len = int(max_len)
        H = self.hidden = self.blocks[0].hidden
        nh, nkv, hd = attn.heads, attn.kv_heads, attn.head_dim
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)

        def w(*shape):
            return (torch.randn(*shape, generator=g, device=self.device) * 0.02).to(torch.bfloat16)

        self.embed = w(attn.vocab, H)
        self.lm_head = w(attn.vocab, H)
        # q, k and v of a layer in one matrix [(nh + 2 nkv) hd, H]; o [H, nh hd]
        self.wqkv = [w((nh + 2 * nkv) * hd, H) for _ in self.blocks]
        self.wo = [w(H, nh * hd) for _ in self.blocks]
        L = len(self.blocks)
        self.k_cache = torch.zeros(L, nkv, self.max_len, hd, dtype=torch.bfloat16, device=self.device)
        self.v_cache = torch.zeros_like(self.k_cache)
        inv = 1.0 / (attn.rope_theta ** (torch.arange(0, hd, 2, device=self.device,
                                                      dtype=torch.float32) / hd))
        ang = torch.arange(self.max_len, device=self.device, dtype=torch.float32)[:, None] * inv
        self.cos, self.sin = torch.cos(ang), torch.sin(ang)      # [max_len, hd / 2]
        self.pos = 0

    # -- pieces ---------------------------------------------------------------
    def _norm(self, h):
        return F.rms_norm(h, (h.shape[-1],), eps=self.cfg.eps)

    def _rope(self, t, p0: int):
        """Rotary embedding of t [heads, T, hd] at positions p0.. (rotate-half form)."""
        T, half = t.shape[1], t.shape[2] // 2
        c = self.cos[p0:p0 + T][None].to(t.dtype)
        s = self.sin[p0:p0 + T][None].to(t.dtype)
        a, b = t[..., :half], t[..., half:]
        return torch.cat((a * c - b * s, b * c + a * s), dim=-1)

    def _attention(self, li: int, h, p0: int):
        """Self-attention of h [T, H] at positions p0..p0+T-1 over the cache; returns [T, H]."""
        c = self.cfg
        T = h.shape[0]
        nh, nkv, hd = c.heads, c.kv_heads, c.head_dim
        qkv = self._norm(h) @ self.wqkv[li].T
        q, k, v = qkv.split((nh * hd, nkv * hd, nkv * hd), dim=-1)
        if c.qk_norm:
            q, k = self._norm(q), self._norm(k)
        q = self._rope(q.reshape(T, nh, hd).transpose(0, 1), p0)
        k = self._rope(k.reshape(T, nkv, hd).transpose(0, 1), p0)
        self.k_cache[li, :, p0:p0 + T] = k
        self.v_cache[li, :, p0:p0 + T] = v.reshape(T, nkv, hd).transpose(0, 1)
        keys = self.k_cache[li, :, :p0 + T][None]
        vals = self.v_cache[li, :, :p0 + T][None]
        with sdpa_kernel(_SDPA_BACKENDS):
            o = F.scaled_dot_product_attention(q[None], keys, vals, is_causal=T > 1 and p0 == 0,
                                               enable_gqa=nkv != nh)
        return o[0].transpose(0, 1).reshape(T, nh * hd) @ self.wo[li].T

    def _layer(self, li: int, h, p0: int):
        h = h + self._attention(li, h, p0)
        blk = self.blocks[li]
        return blk(self._norm(h), residual=h)

    def _logits(self, h_last):
        return self._norm(h_last) @ self.lm_head.T

    # -- the loop ---------------------------------------------------------------
    def reset(self):
        self.pos = 0

    @torch.no_grad()
    def prefill(self, tokens: torch.Tensor, layer_scope=None, logits: bool = False) -> torch.Tensor:
        """Run the prompt ``tokens`` (int64 [T] on the device) layer-major; returns the
        greedy next token ([1] int64, on the device), or with ``logits`` the last position's
        logits ([1, vocab] bf16).  ``layer_scope(li)``, when given, is entered around each
        layer (``StreamHandle.prefill_layer``)."""
        T = tokens.shape[0]
        if T > 1 and self.pos != 0:
            raise ValueError("a multi-token prefill starts at position 0 (reset() first)")
        if self.pos + T > self.max_len:
            raise ValueError(f"prompt of {T} past the cache's {self.max_len} positions")
        h = self.embed[tokens]
        for li in range(len(self.blocks)):
            if layer_scope is not None:
                with layer_scope(li):
                    h = self._layer(li, h, self.pos)
            else:
                h = self._layer(li, h, self.pos)
        self.pos += T
        out = self._logits(h[-1:])
        return out if logits else out.argmax(dim=-1)

    @torch.no_grad()
    def step(self, token: torch.Tensor, logits: bool = False) -> torch.Tensor:
        """One greedy decode step: token [1] -> the next token [1] (both on the device), or
        with ``logits`` the step's logits ([1, vocab] bf16)."""
        if self.pos >= self.max_len:
            raise ValueError(f"the cache's {self.max_len} positions are full")
        h = self.embed[token]
        for li in range(len(self.blocks)):
            h = self._layer(li, h, self.pos)
        self.pos += 1
        out = self._logits(h)
        return out if logits else out.argmax(dim=-1)

    @torch.no_grad()
    def generate(self, prompt: torch.Tensor, steps: int, layer_scope=None) -> torch.Tensor:
        """Greedy decode of ``steps`` tokens after ``prompt``; returns them as int64 [steps]."""
        out = torch.empty(steps, dtype=torch.int64, device=self.device)
        tok = self.prefill(prompt, layer_scope)
        for i in range(steps):
            out[i] = tok[0]
            if i + 1 < steps:
                tok = self.step(tok)
        return out
