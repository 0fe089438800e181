"""MLX affine quantisation format, restated in numpy.  TEST INFRASTRUCTURE ONLY.

Format (bigrig_engine/stream.py:144-151 ``quant`` block; the OLMoE manifest
data/blobs/OLMoE-1B-7B-0125-4bit.experts.manifest.json gives gate_proj weight
[1024, 256] uint32 and scales/biases [1024, 32] float16 for in=2048):

* A weight matrix ``W[out, in]`` is cut into groups of ``group_size`` (64)
  consecutive input elements per output row.
* Each group stores an unsigned code ``q`` in ``[0, 2**bits - 1]`` per element,
  one ``scale`` and one ``bias`` (fp16 or bf16), and ``w = scale * q + bias``.
* Codes are packed as one little-endian bit stream per row: element ``j`` of a row
  sits at bits ``[j*bits, (j+1)*bits)`` of the row's uint32 words read as a
  little-endian stream.  At 4 and 8 bits that is 8 and 4 codes a word; at 3 bits a
  row of ``in`` codes is ``in*3/32`` words and codes straddle words (the shipped
  Qwen3-30B-A3B-3bit manifest gives gate_proj weight [768, 192] for in=2048).  The
  3-bit stream order is this restatement's reading of that layout: no reference
  test or fixture pins it, and MLX is not available to run.

Half-precision values are carried as raw uint16 bit patterns so that bf16 (no
numpy dtype) and fp16 take the same path.

Dequantisation is defined here as ``round_to_dtype(f32(scale) * q + f32(bias))``
with one round-to-nearest-even into the scale dtype.  ``scale * q`` is exact in
fp32 (11- or 8-bit significand times an 8-bit code), so fused and unfused
multiply-add agree, and the CUDA dequant kernel reproduces it bit for bit.
Quantisation (used only to build fixtures) is the documented MLX affine rule:
per group ``scale = (max - min) / (2**bits - 1)``, ``bias = min``,
``q = round((w - bias) / scale)`` clipped to the code range.
"""
from __future__ import annotations

import numpy as np

HALF_DTYPES = ("float16", "bfloat16")


# ----------------------------------------------------------------- half helpers
def f32_to_bf16_bits(a) -> np.ndarray:
    """Round fp32 to bf16 (nearest, ties to even), returned as uint16 bits."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    nan = np.isnan(a)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_half_bits(a, dtype: str) -> np.ndarray:
    """fp32 -> raw bits of ``dtype`` ("float16" or "bfloat16"), round to nearest even."""
    if dtype == "bfloat16":
        return f32_to_bf16_bits(a)
    if dtype == "float16":
        return np.asarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)
    raise ValueError(f"unsupported half dtype {dtype!r}")


def half_bits_to_f32(b, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return bf16_bits_to_f32(b)
    if dtype == "float16":
        return np.asarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)
    raise ValueError(f"unsupported half dtype {dtype!r}")


def bf16_round(a) -> np.ndarray:
    """fp32 values rounded through bf16 and back (the storage rounding of a bf16 tensor)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


# ----------------------------------------------------------------- packing
def codes_per_word(bits: int) -> int:
    if bits not in (4, 8):
        raise ValueError(f"bits must be 4 or 8, got {bits}")
    return 32 // bits


SUPPORTED_BITS = (3, 4, 8)


def pack_codes(q: np.ndarray, bits: int) -> np.ndarray:
    """[out, in] codes -> [out, in*bits/32] uint32, one little-endian bit stream per row."""
    if bits not in SUPPORTED_BITS:
        raise ValueError(f"bits must be one of {SUPPORTED_BITS}, got {bits}")
    q = np.asarray(q, dtype=np.uint32)
    out_dim, in_dim = q.shape
    if (in_dim * bits) % 32:
        raise ValueError(f"in={in_dim} codes of {bits} bits do not fill whole 32-bit words")
    planes = ((q[:, :, None] >> np.arange(bits, dtype=np.uint32)) & 1).astype(np.uint8)
    stream = np.packbits(planes.reshape(out_dim, in_dim * bits), axis=1, bitorder="little")
    return np.ascontiguousarray(stream).view("<u4").astype(np.uint32)


def unpack_codes(words: np.ndarray, bits: int) -> np.ndarray:
    """[out, in*bits/32] uint32 -> [out, in] uint32 codes (the inverse of pack_codes)."""
    if bits not in SUPPORTED_BITS:
        raise ValueError(f"bits must be one of {SUPPORTED_BITS}, got {bits}")
    words = np.ascontiguousarray(np.asarray(words, dtype=np.uint32).astype("<u4"))
    out_dim = words.shape[0]
    planes = np.unpackbits(words.view(np.uint8).reshape(out_dim, -1), axis=1, bitorder="little")
    planes = planes.reshape(out_dim, -1, bits).astype(np.uint32)
    return (planes << np.arange(bits, dtype=np.uint32)).sum(axis=-1, dtype=np.uint32)


# ----------------------------------------------------------------- quantise / dequantise
def quantize(w: np.ndarray, group_size: int = 64, bits: int = 4, scale_dtype: str = "float16"):
    """fp32 ``w[out, in]`` -> (codes uint32 [out, in*bits/32], scales, biases) with
    scales/biases as raw half bits ``[out, in/group_size]`` of ``scale_dtype``."""
    w = np.asarray(w, dtype=np.float32)
    out_dim, in_dim = w.shape
    if in_dim % group_size:
        raise ValueError(f"in={in_dim} is not a multiple of group_size={group_size}")
    g = w.reshape(out_dim, in_dim // group_size, group_size)
    wmax = g.max(axis=-1)
    wmin = g.min(axis=-1)
    n_bins = (1 << bits) - 1
    scale = np.maximum((wmax - wmin) / np.float32(n_bins), np.float32(1e-7)).astype(np.float32)
    s_bits = f32_to_half_bits(scale, scale_dtype)
    b_bits = f32_to_half_bits(wmin, scale_dtype)
    s = half_bits_to_f32(s_bits, scale_dtype)[..., None]
    b = half_bits_to_f32(b_bits, scale_dtype)[..., None]
    q = np.clip(np.rint((g - b) / s), 0, n_bins).astype(np.uint32).reshape(out_dim, in_dim)
    return pack_codes(q, bits), s_bits, b_bits


def dequantize_f32(codes, scales_bits, biases_bits, group_size: int, bits: int,
                   scale_dtype: str) -> np.ndarray:
    """Exact fp32 value of ``scale*q + bias`` per element (one fp32 rounding of the add)."""
    q = unpack_codes(codes, bits).astype(np.float32)
    out_dim, in_dim = q.shape
    s = half_bits_to_f32(scales_bits, scale_dtype).astype(np.float32)
    b = half_bits_to_f32(biases_bits, scale_dtype).astype(np.float32)
    q = q.reshape(out_dim, in_dim // group_size, group_size)
    return (q * s[..., None] + b[..., None]).astype(np.float32).reshape(out_dim, in_dim)


def dequantize(codes, scales_bits, biases_bits, group_size: int, bits: int,
               scale_dtype: str) -> np.ndarray:
    """Dequantised weights as raw bits of ``scale_dtype`` (the ``mx.dequantize`` output dtype)."""
    return f32_to_half_bits(dequantize_f32(codes, scales_bits, biases_bits, group_size, bits,
                                           scale_dtype), scale_dtype)
