"""Seeded synthetic MoE layers for the parity tests: oracle-quantised experts packed into
an HBM slab, plus the oracle's fp32 view of the same bytes.  Test infrastructure."""
from __future__ import annotations

import numpy as np
import torch

from oracle import affine, moe
from bigrig_b200 import formats


class Layer:
    """E experts of an (H, I) SwiGLU layer, weights N(0, std) quantised to the affine format."""

    def __init__(self, H, I, E, bits=4, scale_dtype="float16", seed=0, std=0.02, device="cuda",
                 slot_order=None, plain=False, bias=False, bias_dtype="bfloat16", order=None,
                 activation="silu"):
        self.H, self.I, self.E, self.bits, self.sd = H, I, E, bits, scale_dtype
        self.activation = activation
        self.spec = formats.make_spec(H, I, bits, 64, scale_dtype, plain=plain, bias=bias,
                                      bias_dtype=bias_dtype, order=order)
        self.layout = formats.layout_from_spec(self.spec, {"bits": bits, "group_size": 64,
                                                           "mode": "affine"}
                                               ).with_activation(activation)
        rng = np.random.default_rng(seed)
        self.q, self.bias = {}, {}
        blobs = []
        for e in range(E):
            parts, qe, be = {}, {}, {}
            for p in self.spec:
                o, i = (H, I) if p in ("down_proj", "fc2") else (I, H)
                w = (rng.standard_normal((o, i), dtype=np.float32) * std).astype(np.float32)
                codes, s, b = affine.quantize(w, 64, bits, scale_dtype)
                qe[p] = (codes, s, b)
                parts[p] = {"weight": codes, "scales": s, "biases": b}
                if bias:
                    v = (rng.standard_normal(o).astype(np.float32) * 0.5).astype(np.float32)
                    if bias_dtype == "float32":
                        parts[p]["bias"], be[p] = v, v
                    else:
                        bits16 = affine.f32_to_half_bits(v, bias_dtype)
                        parts[p]["bias"] = bits16
                        be[p] = affine.half_bits_to_f32(bits16, bias_dtype)
            self.q[e] = qe
            self.bias[e] = be
            blobs.append(formats.pack_expert(parts, self.spec))
        self.blobs = blobs
        order = list(range(E)) if slot_order is None else list(slot_order)
        self.slot_of = {e: s for s, e in enumerate(order)}
        slab = np.zeros((E, self.layout.slot_stride), dtype=np.uint8)
        for e in range(E):
            slab[self.slot_of[e], :self.layout.bytes_per_expert] = blobs[e]
        self.slab = torch.from_numpy(slab).to(device)
        self.g2s = torch.tensor([self.slot_of[e] for e in range(E)], dtype=torch.int32,
                                device=device)
        self._w = {}

    def weights(self, e, weight_round=None):
        key = (e, weight_round)
        if key not in self._w:
            self._w[key] = moe.expert_weights_f32(self.q[e], 64, self.bits, self.sd, weight_round)
        return self._w[key]

    def oracle_switch(self, x_f32, idx, weight_round=None, intermediate="h_bf16"):
        return moe.switch_glu(x_f32, idx, lambda e: self.weights(e, weight_round), intermediate,
                              bias_of=lambda e: self.bias[e], activation=self.activation)

    def gemm_rounding(self):
        """(weight_round, intermediate) of the grouped GEMM for this format: 4-bit experts
        compute in their scale dtype (fp16 weights and h for fp16 scales), 8-bit in bf16."""
        if self.bits == 4 and self.sd == "float16":
            return "f16", "h_f16"
        return "bf16", "h_bf16"


def bf16_tensor(a: np.ndarray, device="cuda") -> torch.Tensor:
    bits = affine.f32_to_bf16_bits(a)
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)


def to_f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def random_routing(T, k, E, rng):
    return np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)


def exceedance(got, want, rtol=1e-2, atol=2e-3) -> dict:
    """How far ``got`` is from ``want`` under the bar |got - want| <= atol + rtol * |want|:
    the number of elements outside it, the largest error and the largest error as a
    multiple of that element's allowance."""
    got = np.asarray(got, dtype=np.float32)
    want = np.asarray(want, dtype=np.float32)
    err = np.abs(got - want)
    allow = atol + rtol * np.abs(want)
    return {"outside": int(np.count_nonzero(err > allow)), "of": int(err.size),
            "max_abs": float(err.max()) if err.size else 0.0,
            "max_ratio": float((err / allow).max()) if err.size else 0.0}


# (test id, what was compared, exceedance dict): printed at the end of the run by conftest
EXCEEDANCE_REPORT: list = []


def report(test: str, what: str, r: dict) -> dict:
    """Keep an exceedance result for the end-of-run summary; returns it."""
    EXCEEDANCE_REPORT.append((test, what, r))
    return r


def assert_close(got, want, rtol=1e-2, atol=2e-3):
    """The parity bar for expert outputs, on every element: |got - want| <= atol + rtol * |want|
    (1e-2 relative, 2e-3 absolute, as stated for bf16 expert outputs)."""
    r = exceedance(got, want, rtol, atol)
    assert r["outside"] == 0, (f"{r['outside']} of {r['of']} outside rtol={rtol} atol={atol}; "
                               f"max |d| {r['max_abs']:.3g}, worst {r['max_ratio']:.3g}x the bar")
