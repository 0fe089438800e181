"""The numpy restatement itself: format round trips, dequant rule, router and permutation
semantics, and the packed byte layout against the reference's shipped manifests."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import affine, moe, router
from bigrig_b200 import formats
from bigrig_b200.block import quantize_affine

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("bits", [4, 8])
def test_pack_unpack_roundtrip(bits):
    rng = np.random.default_rng(0)
    q = rng.integers(0, 1 << bits, size=(7, 128)).astype(np.uint32)
    w = affine.pack_codes(q, bits)
    assert w.shape == (7, 128 * bits // 32) and w.dtype == np.uint32
    np.testing.assert_array_equal(affine.unpack_codes(w, bits), q)
    # element j of a word sits at bits [j*bits, (j+1)*bits)
    assert int(w[0, 0]) & ((1 << bits) - 1) == int(q[0, 0])
    assert (int(w[0, 0]) >> bits) & ((1 << bits) - 1) == int(q[0, 1])


@pytest.mark.parametrize("sd", ["float16", "bfloat16"])
@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_dequantize_error_bound(sd, bits):
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((32, 256)) * 0.02).astype(np.float32)
    codes, s, b = affine.quantize(w, 64, bits, sd)
    deq = affine.dequantize_f32(codes, s, b, 64, bits, sd)
    step = affine.half_bits_to_f32(s, sd).repeat(64, axis=1)
    assert np.all(np.abs(deq - w) <= 0.5 * step + np.abs(w) * 2e-2 + 1e-6)


def test_dequant_rule_is_one_rounding():
    # scale * q is exact in fp32, so the half output is round(fp32(s*q + b))
    s = affine.f32_to_half_bits(np.float32(0.0123), "float16")
    b = affine.f32_to_half_bits(np.float32(-0.077), "float16")
    q = np.arange(16, dtype=np.uint32).reshape(1, 16)
    q = np.tile(q, (1, 4))
    codes = affine.pack_codes(q, 4)
    out = affine.dequantize(codes, np.full((1, 1), s, np.uint16), np.full((1, 1), b, np.uint16),
                            64, 4, "float16")
    sf = np.float16(np.uint16(s).view(np.float16)).astype(np.float64)
    bf = np.float16(np.uint16(b).view(np.float16)).astype(np.float64)
    exact = (sf * q.astype(np.float64) + bf).astype(np.float32).astype(np.float16)
    np.testing.assert_array_equal(out.view(np.float16), exact)


def test_bf16_rounding_ties_to_even():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, np.nan, np.inf], dtype=np.float32)
    bits = affine.f32_to_bf16_bits(x)
    assert bits[0] == 0x3F80 and bits[1] == 0x3F82
    assert bits[3] == 0x7FC0 and bits[4] == 0x7F80
    ref = torch.from_numpy(x[:3]).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(bits[:3], ref)


@pytest.mark.parametrize("sd", ["float16", "bfloat16"])
@pytest.mark.parametrize("bits", [4, 8])
def test_torch_quantizer_equals_restatement(sd, bits):
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((48, 192)) * 0.02).astype(np.float32)
    codes, s, b = affine.quantize(w, 64, bits, sd)
    tw, ts, tb = quantize_affine(torch.from_numpy(w), 64, bits,
                                 torch.float16 if sd == "float16" else torch.bfloat16)
    np.testing.assert_array_equal(tw.numpy().view(np.uint32), codes)
    np.testing.assert_array_equal(ts.view(torch.int16).numpy().view(np.uint16), s)
    np.testing.assert_array_equal(tb.view(torch.int16).numpy().view(np.uint16), b)


def test_router_modes_and_ties():
    lg = np.array([[0.5, 2.0, 2.0, -1.0, 3.0, 0.0]], dtype=np.float32)
    idx, sc = router.topk(lg, 3, "softmax_topk")
    assert idx.tolist() == [[4, 1, 2]]                    # ties to the lower id
    p = router.softmax(lg)
    np.testing.assert_allclose(sc, p[:, [4, 1, 2]], rtol=1e-6)
    _, scn = router.topk(lg, 3, "softmax_topk", norm_topk=True)
    np.testing.assert_allclose(scn.sum(), 1.0, rtol=1e-6)
    idx2, sc2 = router.topk(lg, 2, "topk_softmax")
    assert idx2.tolist() == [[4, 1]]
    np.testing.assert_allclose(sc2, router.softmax(np.array([[3.0, 2.0]], np.float32)), rtol=1e-6)
    with pytest.raises(ValueError):
        router.topk(lg, 7)


def test_permutation_semantics():
    idx = np.array([[3, 1], [1, 0], [3, 2]])
    p = router.permutation(idx, 4)
    assert p["order"].tolist() == [3, 1, 2, 5, 0, 4]
    assert p["tok"].tolist() == [1, 0, 1, 2, 0, 2]
    assert p["rank"].tolist() == [1, 1, 0, 1, 0, 0]
    np.testing.assert_array_equal(p["order"][p["inv"]], np.arange(6))
    assert p["offsets"].tolist() == [0, 1, 3, 4, 6]
    assert p["seg_expert"].tolist() == [0, 1, 2, 3]


def test_expert_forward_matches_by_hand_formula():
    # the reference's by-hand oracle (tests/test_plan_invariance.py:149-160), fp32 throughout
    rng = np.random.default_rng(4)
    H, I = 128, 64
    ws = {}
    for p in moe.PROJ:
        o, i = (H, I) if p == "down_proj" else (I, H)
        ws[p] = affine.quantize((rng.standard_normal((o, i)) * 0.05).astype(np.float32), 64, 4,
                                "bfloat16")
    w = moe.expert_weights_f32(ws, 64, 4, "bfloat16")
    x = affine.bf16_round(rng.standard_normal((3, H)).astype(np.float32))
    ref = (moe.silu(x @ w["gate_proj"].T) * (x @ w["up_proj"].T)) @ w["down_proj"].T
    got = moe.expert_forward(x, w)
    got32 = moe.expert_forward(x, w, "f32")
    got16 = moe.expert_forward(x, w, "bf16")
    assert np.abs(got - ref).max() / np.abs(ref).max() < 0.02
    np.testing.assert_allclose(got, got32, rtol=1e-2, atol=2e-3)
    np.testing.assert_allclose(got, got16, rtol=1e-2, atol=2e-3)


def test_spec_matches_shipped_manifests():
    with open(os.path.join(GOLD, "manifest_golden.json")) as f:
        m = json.load(f)
    ol = m["OLMoE-1B-7B-0125-4bit"]
    spec = formats.make_spec(2048, 1024, 4, 64, "float16")
    assert spec == ol["layer0"]["spec"]
    assert formats.bytes_per_expert(spec) == ol["layer0"]["bytes_per_expert"] == 3538944
    assert ol["n_layers"] * 64 * 3538944 == ol["total_bytes"]
    regions = formats.manifest_regions({"regions": ol["regions_head"]})
    assert regions[(0, 1)] == (3538944, 3538944)
    L = formats.layout_from_spec(spec, ol["layer0"]["quant"])
    assert (L.hidden, L.inter, L.bits) == (2048, 1024, 4)
    assert L.weight_off == (0, 1179648, 2359296)
    assert L.scales_off == (1048576, 2228224, 3407872)
    # the 3-bit manifest: its spec is make_spec's at 3 bits, and the layout the kernels
    # read is the widened 4-bit one, fed from the 3-bit bytes the blob stores
    q3 = m["Qwen3-30B-A3B-3bit"]["layer0"]
    spec3 = formats.make_spec(2048, 768, 3, 64, "bfloat16")
    assert spec3 == q3["spec"]
    assert formats.bytes_per_expert(spec3) == q3["bytes_per_expert"]
    L3 = formats.layout_from_spec(q3["spec"], q3["quant"])
    assert (L3.bits, L3.source_bits, L3.source_bytes) == (4, 3, q3["bytes_per_expert"])
    L4 = formats.layout_from_spec(formats.make_spec(2048, 768, 4, 64, "bfloat16"),
                                  {"bits": 4, "group_size": 64, "mode": "affine"})
    assert (L3.weight_off, L3.scales_off, L3.slot_stride) == (L4.weight_off, L4.scales_off, L4.slot_stride)
    with pytest.raises(NotImplementedError):
        formats.layout_from_spec(formats.make_spec(2048, 768, 4, 64, "bfloat16"),
                                 {"bits": 2, "group_size": 64, "mode": "affine"})


def test_pack_unpack_expert_roundtrip():
    spec = formats.make_spec(128, 64, 8, 64, "bfloat16")
    rng = np.random.default_rng(5)
    arrays = {p: {c: rng.integers(0, 2 ** 16, size=meta["shape"]).astype(
        np.uint32 if meta["dtype"] == "uint32" else np.uint16) for c, meta in spec[p].items()}
        for p in spec}
    blob = formats.pack_expert(arrays, spec)
    assert blob.nbytes == formats.bytes_per_expert(spec)
    back = formats.unpack_expert(blob, spec)
    for p in spec:
        for c in spec[p]:
            np.testing.assert_array_equal(back[p][c], arrays[p][c])
    with pytest.raises(ValueError):
        formats.unpack_expert(blob[:-1], spec)


def test_three_bit_codes_straddle_words():
    """3-bit codes as one little-endian bit stream per row: 32 codes fill 3 words, code
    10 spans bits 30-32 (words 0 and 1), and packing inverts unpacking."""
    q = np.zeros((1, 32), dtype=np.uint32)
    q[0, 10] = 0b101                                   # bits 30, 32
    w = affine.pack_codes(q, 3)
    assert w.shape == (1, 3)
    assert int(w[0, 0]) == 1 << 30 and int(w[0, 1]) == 1 and int(w[0, 2]) == 0
    rng = np.random.default_rng(9)
    q = rng.integers(0, 8, size=(7, 128)).astype(np.uint32)
    assert np.array_equal(affine.unpack_codes(affine.pack_codes(q, 3), 3), q)
    # a 3-bit code is the same 4-bit code: widening repacks without changing a weight
    w3 = rng.standard_normal((4, 128)).astype(np.float32) * 0.02
    c3, s, b = affine.quantize(w3, 64, 3, "bfloat16")
    c4 = affine.pack_codes(affine.unpack_codes(c3, 3), 4)
    assert np.array_equal(affine.dequantize(c3, s, b, 64, 3, "bfloat16"),
                          affine.dequantize(c4, s, b, 64, 4, "bfloat16"))


# ------------------------------------------------------------------ expert shapes
def test_plain_and_bias_layouts():
    """fc1/fc2 experts and the affine bias, components in any packed order
    (reference tests/test_fast_decode.py:95-110)."""
    from bigrig_b200 import formats
    q = {"bits": 4, "group_size": 64, "mode": "affine"}
    order = ("biases", "bias", "scales", "weight")
    s = formats.make_spec(256, 128, 4, 64, "bfloat16", plain=True, bias=True, order=order)
    assert tuple(s) == ("fc1", "fc2") and tuple(s["fc1"]) == order
    L = formats.layout_from_spec(s, q)
    assert L.plain and L.has_bias and L.activation == 0
    offs = formats.component_offsets(s)
    assert L.weight_off == (offs[("fc1", "weight")], 0, offs[("fc2", "weight")])
    assert L.bias_off == (offs[("fc1", "bias")], 0, offs[("fc2", "bias")])
    assert L.bytes_per_expert == formats.bytes_per_expert(s)
    assert L.with_activation("relu2").activation == 2
    with pytest.raises(NotImplementedError):
        L.with_activation("gpt_oss")              # gated only
    G = formats.layout_from_spec(formats.make_spec(256, 128, 8, 64, bias=True,
                                                   bias_dtype="float32"),
                                 {"bits": 8, "group_size": 64})
    assert not G.plain and G.has_bias and (G.flags >> 2) & 3 == 0
    assert G.with_activation("gpt_oss").activation == 1
    with pytest.raises(NotImplementedError):
        G.with_activation("relu2")                # plain only
    # a bias on some projections only is refused
    half = formats.make_spec(256, 128, bias=True)
    del half["up_proj"]["bias"]
    with pytest.raises(NotImplementedError):
        formats.layout_from_spec(half, q)
    # pack / unpack round trip in the listed order
    rng = np.random.default_rng(0)
    arrays = {p: {c: rng.integers(0, 2**15, size=m["shape"]).astype(
        np.uint32 if m["dtype"] == "uint32" else np.uint16) for c, m in s[p].items()} for p in s}
    blob = formats.pack_expert(arrays, s)
    back = formats.unpack_expert(blob, s)
    for p in s:
        for c in s[p]:
            np.testing.assert_array_equal(back[p][c], arrays[p][c])


def test_variant_activations():
    from oracle import moe as omoe
    g = np.array([-9.0, -1.0, 0.0, 3.0, 8.0], dtype=np.float32)
    u = np.array([-8.0, 0.5, 2.0, -3.0, 9.0], dtype=np.float32)
    np.testing.assert_allclose(omoe.act_gated(g, u, "silu"), g / (1 + np.exp(-g)) * u, rtol=1e-6)
    gc, uc = np.minimum(g, 7), np.clip(u, -7, 7)
    np.testing.assert_allclose(omoe.act_gated(g, u, "gpt_oss"),
                               gc / (1 + np.exp(-1.702 * gc)) * (uc + 1), rtol=1e-6)
    np.testing.assert_array_equal(omoe.act_plain(g, "relu2"), np.maximum(g, 0) ** 2)
    # a plain expert with biases: fc2(act(fc1 x + b1)) + b2
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 64)).astype(np.float32)
    w = {"fc1": rng.standard_normal((32, 64)).astype(np.float32) * 0.1,
         "fc2": rng.standard_normal((64, 32)).astype(np.float32) * 0.1}
    b = {"fc1": rng.standard_normal(32).astype(np.float32), "fc2": rng.standard_normal(64).astype(np.float32)}
    y = omoe.expert_forward(x, w, "f32", b, "relu2")
    h = np.maximum(x @ w["fc1"].T + b["fc1"], 0) ** 2
    np.testing.assert_allclose(y, h @ w["fc2"].T + b["fc2"], rtol=1e-2, atol=1e-2)
