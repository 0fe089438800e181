"""SwiGLU expert layer over MLX-affine experts, restated in numpy.  TEST INFRASTRUCTURE ONLY.

Follows the reference's by-hand oracle (tests/test_plan_invariance.py:149-160):
``y = (silu(x . Wg^T) * (x . Wu^T)) . Wd^T`` per (token, expert) pair, with the
weights dequantised from their affine codes, and the per-expert call order of
``_forward_views_one`` (bigrig_engine/stream.py:1278-1318): up, gate,
``act(up, gate) = silu(gate) * up``, down.  The layer returns the pairs
unreduced, ``y[..., k, H]`` (bigrig_engine/stream.py:1523-1525); the caller's
MoE block applies ``sum_k score_k * y_k``.

Rounding points: gate and up stay in fp32 (the accumulator), the activation
``h = silu(gate) * up`` is stored as bf16 (the input dtype of the down
projection), and the output is bf16.  ``intermediate="bf16"`` also rounds gate
and up to bf16 (a model whose projections emit bf16), ``"f32"`` keeps h in fp32
too, ``"h_f16"`` stores h as fp16 (an fp16 model's down-projection input); all
agree within the 1e-2 relative / 2e-3 absolute tolerance of the
parity tests on typical rows.  The default is the one the kernels implement:
rounding gate/up before the SiLU lets a one-ulp flip of a large gate value move a
whole output row, which no reduction order can reproduce bit for bit.
"""
from __future__ import annotations

import numpy as np

from .affine import bf16_round, dequantize_f32, f32_to_half_bits, half_bits_to_f32

PROJ = ("gate_proj", "up_proj", "down_proj")
PLAIN = ("fc1", "fc2")          # the plain two-layer expert fc2(act(fc1(x))) (stream.py:56-76)


def f16_round(a) -> np.ndarray:
    """fp32 values rounded through fp16 and back (round to nearest even)."""
    return half_bits_to_f32(f32_to_half_bits(np.asarray(a, dtype=np.float32), "float16"), "float16")


def silu(g: np.ndarray) -> np.ndarray:
    g = g.astype(np.float32)
    return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)


def expert_weights_f32(expert: dict, group_size: int, bits: int, scale_dtype: str,
                       weight_round: str | None = None) -> dict:
    """{proj: fp32 [out, in]} for one expert given {proj: (codes, scales_bits, biases_bits)}.

    ``weight_round="bf16"`` rounds each dequantised weight to bf16 once, as a
    multi-row quantized matmul does when it dequantises a weight tile into the
    activation dtype before the matrix product; ``"f16"`` rounds it to fp16 once (the
    ``mx.dequantize`` value of an fp16-scaled format, the operand of an fp16 model's
    matrix product); None keeps the exact fp32 value, as the one-row (GEMV) form
    ``s * sum(q x) + b * sum(x)`` effectively uses."""
    out = {p: dequantize_f32(*expert[p][:3], group_size, bits, scale_dtype) for p in expert}
    if weight_round == "bf16":
        out = {p: bf16_round(w) for p, w in out.items()}
    elif weight_round == "f16":
        out = {p: f16_round(w) for p, w in out.items()}
    elif weight_round is not None:
        raise ValueError(f"weight_round must be None, 'bf16' or 'f16', got {weight_round!r}")
    return out


def act_gated(gate: np.ndarray, up: np.ndarray, activation: str = "silu") -> np.ndarray:
    """The gated expert's activation: SwiGLU ``silu(gate) * up`` (stream.py:1163-1166), or
    gpt-oss's clamped form (the gpt-oss model's own SwiGLU, from its published model code;
    mlx_lm's module is not in the reference tree): g = min(gate, 7), u = clip(up, -7, 7),
    ``g * sigmoid(1.702 g) * (u + 1)``."""
    if activation in ("silu", "swiglu"):
        return (silu(gate) * up).astype(np.float32)
    if activation == "gpt_oss":
        g = np.minimum(gate, np.float32(7.0)).astype(np.float32)
        u = np.clip(up, np.float32(-7.0), np.float32(7.0)).astype(np.float32)
        sig = (np.float32(1.0) / (np.float32(1.0) + np.exp(np.float32(-1.702) * g))).astype(np.float32)
        return (g * sig * (u + np.float32(1.0))).astype(np.float32)
    raise ValueError(f"gated activation {activation!r}")


def act_plain(h: np.ndarray, activation: str = "silu") -> np.ndarray:
    """The plain expert's activation of fc1's output (stream.py:1167-1169): SiLU, or
    squared ReLU ``max(h, 0)^2``."""
    if activation == "silu":
        return silu(h)
    if activation == "relu2":
        r = np.maximum(h, np.float32(0.0)).astype(np.float32)
        return (r * r).astype(np.float32)
    raise ValueError(f"plain activation {activation!r}")


def expert_forward(x: np.ndarray, w: dict, intermediate: str = "h_bf16", bias: dict | None = None,
                   activation: str = "silu") -> np.ndarray:
    """x fp32 [R, H] (values of a bf16 tensor) -> y fp32 [R, H] (values of bf16).

    ``w`` holds gate_proj/up_proj/down_proj (gated) or fc1/fc2 (plain) as fp32 ``[out, in]``;
    ``bias`` the projections' affine biases ``[out]`` (fp32 values), added to each
    projection's fp32 output (stream.py:79-81)."""
    if intermediate not in ("h_bf16", "h_f16", "bf16", "f32"):
        raise ValueError(f"intermediate must be h_bf16, h_f16, bf16 or f32, got {intermediate!r}")
    keep = lambda a: a.astype(np.float32)  # noqa: E731
    rnd_gu = bf16_round if intermediate == "bf16" else keep
    rnd_h = keep if intermediate == "f32" else f16_round if intermediate == "h_f16" else bf16_round
    b = bias or {}

    def proj(name, a):
        out = (a @ w[name].T).astype(np.float32)
        if name in b:
            out = (out + np.asarray(b[name], dtype=np.float32)).astype(np.float32)
        return out

    if "fc1" in w:
        h = rnd_h(act_plain(rnd_gu(proj("fc1", x)), activation))
        return bf16_round(proj("fc2", h))
    up = rnd_gu(proj("up_proj", x))
    gate = rnd_gu(proj("gate_proj", x))
    h = rnd_h(act_gated(gate, up, activation))
    return bf16_round(proj("down_proj", h))


def switch_glu(x: np.ndarray, indices: np.ndarray, weights_of, intermediate: str = "h_bf16",
               bias_of=None, activation: str = "silu"):
    """Unreduced expert outputs.  x [T, H] fp32, indices [T, k] int -> y [T, k, H] fp32.

    ``weights_of(e)`` returns the fp32 weight dict of expert ``e``.  Pairs are
    grouped by expert (each expert's weights dequantised once) and written back
    in the caller's (token, k) order, which is what the inverse permutation of
    bigrig_engine/stream.py:1246-1276 achieves.
    """
    T, k = indices.shape
    H = x.shape[1]
    y = np.zeros((T, k, H), dtype=np.float32)
    flat = indices.reshape(-1)
    for e in np.unique(flat):
        pos = np.nonzero(flat == e)[0]
        rows = x[pos // k]
        y.reshape(T * k, H)[pos] = expert_forward(
            rows, weights_of(int(e)), intermediate,
            bias_of(int(e)) if bias_of is not None else None, activation)
    return y


def combine(y: np.ndarray, scores: np.ndarray) -> np.ndarray:
    """sum_k score[t, k] * y[t, k, :] accumulated in fp32 in k order, stored as bf16."""
    T, k, H = y.shape
    acc = np.zeros((T, H), dtype=np.float32)
    for j in range(k):
        acc = (acc + scores[:, j:j + 1].astype(np.float32) * y[:, j, :]).astype(np.float32)
    return bf16_round(acc)
