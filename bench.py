"""Benchmark of the MoE expert hot path on B200 -- one JSON line on rank 0.

Workload (the OLMoE-1B-7B-shaped decode): the model's 16
MoE layers (hidden 2048, 64 experts, top-8, SwiGLU intermediate 1024, MLX affine
4-bit g64 with fp16 scales/biases, router N(0, 0.02) bf16 plus a per-expert
N(0, 1) bias), batch-1 greedy-decode shape, each layer's expert pool capped at 16
of 64 experts in HBM and refilled from pinned host DRAM on a side stream (LFUDA).
A step is one token through all 16 MoE layers: router logits, warp-shuffle top-k
+ softmax, the pool's ensure (host readback of the routing, as the reference's),
the fused dequantising GEMVs and the combine, plus the residual add.  Attention,
embeddings and the LM head are not part of the hot path and are not run.  Inputs
are seeded synthetic token embeddings, N(0, 1) bf16 -- no dataset exists here.

Also reported (outside the K timed steps): the 2048-token prompt through the
capped stack in layer-major order (prefill tok/s), the same decode with every
expert resident (sync-free, one CUDA graph per token: the MoE-layer HBM GB/s and
its fraction of the measured peak), and the CPU restatement's throughput.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Multi-GPU: one process per GPU under torchrun, expert parallel.  Rank r owns the
contiguous block r of every layer's experts (E/N of them, in a pool of
min(16, E/N) slots refilled from its own pinned host store); every rank decodes
its own token stream with the replicated router and sends each routed pair to the
owning rank by NCCL all-to-all (fixed-capacity blocks when the local pool holds
all its experts, exact counts otherwise), which computes it and sends it back for
the combine.  The timed region is bracketed by barriers and the slowest rank's
time is the job's; value = tokens of all ranks / that time ("weak" scaling).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = {"workload": "olmoe-1b-7b MoE stack decode, B=1, pool 16/64 per layer refilled from "
                   "pinned host", "layers": 16, "hidden": 2048, "inter": 1024, "experts": 64,
       "top_k": 8, "bits": 4, "group_size": 64, "scale_dtype": "float16", "capacity": 16,
       "policy": "lfuda", "prompt": 2048, "prefill_chunk": 512, "family": "olmoe"}
METRIC = "decode tok/s (MoE layers of an OLMoE-1B-7B-shaped model, pool 16/64)"


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _bf16_sustained():
    """The sustained bf16 tensor peak (a kernel timed inside a long step), TFLOP/s."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured sustained"
    return 1400.0, "fallback sustained"


# ------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampling every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            vis = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = vis.split(",")[self.idx] if vis else str(self.idx)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={phys}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, IndexError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.remove(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


# the source file of each kernel a traffic figure may be quoted for
KERNEL_SOURCES = {"decode_layer_kernel": "decode_layer.cu", "decode_split_kernel": "decode_split.cu",
                  "gemv_gate_up_kernel": "gemv.cu", "grouped_gemm_kernel": "gemm_sm100.cu"}


def kernel_source_hash(kernel: str) -> str | None:
    """First 12 hex digits of the sha256 of the kernel's source file (csrc/<file>)."""
    import hashlib
    f = KERNEL_SOURCES.get(kernel)
    path = os.path.join(ROOT, "bigrig_b200", "csrc", f) if f else None
    if not path or not os.path.exists(path):
        return None
    return hashlib.sha256(open(path, "rb").read()).hexdigest()[:12]


def _traffic() -> dict:
    """DRAM bytes per launch (read + write) of the profiled kernels, from the ncu summary
    committed in profiles/traffic.txt ("<kernel> <bytes> <source sha256[:12]>" lines).  A
    figure whose recorded source hash differs from the kernel's current source was measured
    on other code: it is left out (the line then carries null), never quoted stale."""
    out = {}
    tpath = os.path.join(ROOT, "profiles", "traffic.txt")
    if os.path.exists(tpath):
        for line in open(tpath):
            parts = line.split()
            if len(parts) >= 3 and not line.startswith("#"):
                if parts[2] != kernel_source_hash(parts[0]):
                    continue
                try:
                    out[parts[0]] = int(float(parts[1]))
                except ValueError:
                    pass
    return out


# ------------------------------------------------------------------ model
def build_model(device, seed: int, experts=None, layers=None):
    """Router weights (replicated on every rank) and a pinned host store holding the
    given global expert ids of every layer (all of them by default)."""
    from bigrig_b200.block import fill_store, make_blocks
    from bigrig_b200.fetch import HostExpertStore
    from bigrig_b200.formats import bytes_per_expert, make_spec
    c = dict(CFG)
    if layers is not None:
        c["layers"] = layers
    blocks = make_blocks(c["layers"], c["hidden"], c["inter"], c["experts"], c["top_k"],
                         c["family"], c["bits"], c["group_size"], c["scale_dtype"], True,
                         seed=seed, device=device)
    spec = make_spec(c["hidden"], c["inter"], c["bits"], c["group_size"], c["scale_dtype"])
    ids = list(range(c["experts"])) if experts is None else list(experts)
    store = HostExpertStore({li: (len(ids), bytes_per_expert(spec)) for li in range(c["layers"])})
    fill_store(store, c["layers"], c["hidden"], c["inter"], c["experts"], c["bits"],
               c["group_size"], c["scale_dtype"], seed=seed + 1, device=device, experts=ids)
    torch.cuda.synchronize(device)
    return blocks, store


def stack_step(blocks, x):
    """One token through every MoE layer: h <- h + moe(h) (the residual add is fused)."""
    h = x
    for blk in blocks:
        h = blk(h, residual=h)
    return h


def algorithmic_layer_bytes(T: int, distinct: int) -> int:
    """Decode MoE layer bytes: U * bytes_per_expert + router E*H*2 + x in / y out."""
    c = CFG
    from bigrig_b200.formats import bytes_per_expert, make_spec
    bpe = bytes_per_expert(make_spec(c["hidden"], c["inter"], c["bits"], c["group_size"],
                                     c["scale_dtype"]))
    return distinct * bpe + c["experts"] * c["hidden"] * 2 + T * c["hidden"] * 2 * 2


# ------------------------------------------------------------------ the other named shapes
# BASELINE configs 3-5, each measured at N=1 as an extra key of the line (never the headline).
SHAPES = {
    "c3": {"name": "qwen3-30b-a3b-shaped", "layers": 48, "hidden": 2048, "inter": 768,
           "experts": 128, "top_k": 8, "bits": 4, "scale_dtype": "bfloat16", "family": "qwen3",
           "prefill": 4096, "decode_batches": (1, 8)},
    "c4": {"name": "gpt-oss-120b-shaped", "layers": 36, "hidden": 2880, "inter": 2880,
           "experts": 128, "top_k": 4, "bits": 4, "scale_dtype": "bfloat16",
           "family": "gpt_oss", "prefill": 8 * 2048, "decode_batches": (64,)},
    "c5": {"name": "mixtral-8x7b-shaped", "layers": 32, "hidden": 4096, "inter": 14336,
           "experts": 8, "top_k": 2, "bits": 8, "scale_dtype": "float16", "family": "mixtral",
           "prefill": 8192, "capacity": 2},
}


def _normed(b):
    """A pre-norm MoE layer, h -> h + moe(rms_norm(h)), as these model families place the
    block behind an RMSNorm (unit weight here): without it a random-init stack of wide
    experts grows its hidden state layer after layer until the logits overflow."""
    H = b.hidden

    def layer(h):
        return b(torch.nn.functional.rms_norm(h, (H,), eps=1e-6), residual=h)
    return layer


def _normed_step(blocks, x):
    h = x
    for b in blocks:
        h = b(torch.nn.functional.rms_norm(h, (b.hidden,), eps=1e-6), residual=h)
    return h


def _expert_bank(dev, sh: dict, seed: int):
    """One layer's worth of distinct experts (N(0, 0.02) quantised on the GPU), slab rows."""
    from bigrig_b200.block import random_expert_bytes
    from bigrig_b200.formats import layout_from_spec, make_spec
    spec = make_spec(sh["hidden"], sh["inter"], sh["bits"], 64, sh["scale_dtype"])
    L = layout_from_spec(spec, {"bits": sh["bits"], "group_size": 64, "mode": "affine"})
    sd = {"float16": torch.float16, "bfloat16": torch.bfloat16}[sh["scale_dtype"]]
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    bank = torch.zeros(sh["experts"], L.slot_stride, dtype=torch.uint8, device=dev)
    for e in range(sh["experts"]):
        bank[e, :L.bytes_per_expert] = random_expert_bytes(sh["hidden"], sh["inter"], sh["bits"],
                                                           64, sd, g, dev)
    return bank, spec, L


def _layer_perm(E: int, li: int) -> torch.Tensor:
    """Which bank expert plays expert e of layer li: a fixed per-layer permutation."""
    return torch.from_numpy(np.random.default_rng(10_000 + li).permutation(E))


def _resident_blocks(dev, sh: dict, seed: int):
    """Every layer's experts resident in its own HBM slab (the bank, permuted per layer)."""
    from bigrig_b200.block import make_blocks
    from bigrig_b200.stream import ExpertPool, StreamingSwitchGLU
    bank, spec, L = _expert_bank(dev, sh, seed)
    blocks = make_blocks(sh["layers"], sh["hidden"], sh["inter"], sh["experts"], sh["top_k"],
                         sh["family"], sh["bits"], 64, sh["scale_dtype"], True, seed=seed + 1,
                         device=dev)
    for b in blocks:
        pool = ExpertPool(b.layer, None, sh["experts"], sh["experts"], spec, quant=b.quant,
                          device=dev)
        pool.adopt(bank.index_select(0, _layer_perm(sh["experts"], b.layer).to(dev)))
        b.switch = StreamingSwitchGLU(pool, None)
        b.switch.refresh()
        pool.g2s_device()
        pool.settle()
    del bank
    return blocks, spec, L


def _decode_bytes(blocks, xs, bpe: int) -> float:
    """Mean algorithmic HBM bytes of one MoE layer over the steps' inputs: distinct routed
    experts x bytes per expert + router weights + tokens in and out, with every layer's
    routing recomputed on the stack's own hidden states."""
    tot, n = 0.0, 0
    for x in xs:
        h = x
        for b in blocks:
            hn = torch.nn.functional.rms_norm(h, (b.hidden,), eps=1e-6)
            idx, _ = b.route(hn)
            U = int(torch.unique(idx).numel())
            tot += U * bpe + b.n_experts * b.hidden * 2 + 2 * h.shape[0] * b.hidden * 2
            n += 1
            h = b(hn, residual=h)
    return tot / max(1, n)


def _graph_decode(dev, blocks, B: int, K: int, W: int, seed: int, bpe: int, peak: float) -> dict:
    """B tokens through the resident stack per step, one CUDA graph per step; K timed steps
    on fresh random inputs.  tok/s and the MoE layers' HBM roofline."""
    from bigrig_b200 import ops
    H = blocks[0].hidden
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    xs = torch.randn(W + K, B, H, generator=g, device=dev).to(torch.bfloat16)
    ws = ops.default_workspace(dev)
    ws.reserve(ops.workspace_bytes(B, blocks[0].top_k, blocks[0].n_experts,
                                   blocks[0].switch._pool.layout))
    xin = xs[0].clone()
    for _ in range(2):
        _normed_step(blocks, xin)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream(device=dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(st):
        _normed_step(blocks, xin)
    torch.cuda.current_stream(dev).wait_stream(st)
    with torch.cuda.graph(graph):
        _normed_step(blocks, xin)
    for i in range(W):
        xin.copy_(xs[i])
        graph.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(K):
        xin.copy_(xs[W + i])
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / K
    del graph
    layer_bytes = _decode_bytes(blocks, [xs[W + i] for i in range(min(K, 4))], bpe)
    layer_ms = ms / len(blocks)
    gbs = layer_bytes / (layer_ms / 1e3) / 1e9
    return {"batch": B, "tok_s": B / (ms / 1e3), "ms_per_step": ms, "steps": K,
            "roofline": {"kernel": "one-token layer kernel (decode_split_kernel where it fits)"
                         if B == 1 else "moe layer (GEMV chain / "
                         "grouped GEMM)", "bound": "hbm", "achieved": gbs, "peak": peak,
                         "unit": "GB/s", "frac": gbs / peak,
                         "bytes_per_layer": layer_bytes, "ms_per_layer": layer_ms,
                         "note": "algorithmic layer bytes (distinct routed experts x bytes per "
                                 "expert + router + tokens) over graph time per layer"}}


def _prefill_gemm(dev, blocks, T: int, seed: int, peak: float, peak_kind: str, layer_scope=None,
                  warm: bool = True) -> dict:
    """A T-token prompt through the stack layer-major, token-wise (each layer once over all
    T tokens); the grouped GEMM's launches timed with CUDA events."""
    from bigrig_b200 import _lib, layered
    H, k, I = blocks[0].hidden, blocks[0].top_k, blocks[0].inter
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    prompt = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    layers = [_normed(b) for b in blocks]
    if warm:
        layered.prefill(layers, [prompt], token_wise=True, layer_scope=layer_scope)
    torch.cuda.synchronize(dev)
    _lib.timing_enable(["gemm_gate_up", "gemm_down"])
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    layered.prefill(layers, [prompt], token_wise=True, layer_scope=layer_scope)
    e1.record()
    torch.cuda.synchronize(dev)
    _lib.timing_enable([])
    gu, _ = _lib.timing_read("gemm_gate_up")
    dn, _ = _lib.timing_read("gemm_down")
    ms = e0.elapsed_time(e1)
    flops = 6.0 * T * k * H * I * len(blocks)
    gemm_s = (gu + dn) / 1e3
    ach = flops / gemm_s / 1e12 if gemm_s > 0 else None
    return {"tokens": T, "tok_s": T / (ms / 1e3), "ms": ms,
            "roofline": {"kernel": "grouped_gemm_kernel", "bound": "tensor", "achieved": ach,
                         "peak": peak, "peak_kind": peak_kind, "unit": "TFLOP/s",
                         "frac": ach / peak if ach else None, "flops": flops,
                         "gemm_ms": gemm_s * 1e3, "gate_up_ms": gu, "down_ms": dn}}


def _h2d_gbs(dev) -> float:
    """Pinned host -> device copy bandwidth, GB/s (1 GiB, best of 3)."""
    src = torch.empty(1 << 30, dtype=torch.uint8).pin_memory()
    dst = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    best = 0.0
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dst.copy_(src, non_blocking=True)
        e1.record()
        torch.cuda.synchronize(dev)
        best = max(best, (1 << 30) / (e0.elapsed_time(e1) / 1e3) / 1e9)
    del src, dst
    return best


def bench_shape(dev, key: str, W: int, hbm_peak: float, hbm_kind: str, bf16_peak: float,
                bf16_kind: str) -> dict:
    """The BASELINE config ``key`` at N=1: resident decode and prefill (c3, c4), or the
    host-streamed pool (c5)."""
    from bigrig_b200.formats import bytes_per_expert
    sh = SHAPES[key]
    out = {"workload": sh["name"], **{k: sh[k] for k in ("layers", "hidden", "inter", "experts",
                                                         "top_k", "bits", "scale_dtype")}}
    t0 = time.perf_counter()
    if key in ("c3", "c4"):
        blocks, spec, L = _resident_blocks(dev, sh, seed=31 + len(key))
        bpe = bytes_per_expert(spec)
        out["resident_gb"] = len(blocks) * sh["experts"] * L.slot_stride / 1e9
        out["data"] = ("one layer's experts N(0,0.02) quantised on the GPU, each layer holding its "
                       "own HBM copy in a per-layer permutation; router N(0,0.02) + bias N(0,1) "
                       "per layer; random bf16 N(0,1) tokens")
        out["decode"] = [_graph_decode(dev, blocks, B, 20, W, 500 + B, bpe, hbm_peak)
                         for B in sh["decode_batches"]]
        for d in out["decode"]:
            d["roofline"]["peak_kind"] = hbm_kind
        out["prefill"] = _prefill_gemm(dev, blocks, sh["prefill"], 77, bf16_peak, bf16_kind)
        del blocks
    else:
        out.update(_bench_streamed(dev, sh, W, hbm_peak, bf16_peak, bf16_kind))
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    out["setup_and_run_s"] = time.perf_counter() - t0
    return out


def _bench_streamed(dev, sh: dict, W: int, hbm_peak: float, bf16_peak: float, bf16_kind: str) -> dict:
    """Config 5: every layer's pool holds ``capacity`` experts in HBM, the rest are copied from
    pinned host DRAM on a side stream (staged ahead from the next layer's router when it
    can).  Prefill token-wise, then a decode sample; copy bandwidth against pinned H2D."""
    from bigrig_b200.block import make_blocks
    from bigrig_b200.fetch import HostExpertStore
    from bigrig_b200.stream import attach
    bank, spec, L = _expert_bank(dev, sh, seed=51)
    E, bpe = sh["experts"], L.bytes_per_expert
    base = bank[:, :bpe].cpu()
    del bank
    torch.cuda.empty_cache()
    # the experts live once per permutation in pinned host DRAM; all layers share two
    # permutations (the copies over PCIe are real, the host bytes are reused)
    perms = [base.index_select(0, _layer_perm(E, j)).pin_memory() for j in range(2)]
    del base
    store = HostExpertStore({}, pin=False)
    store.pinned = True
    store.layers = {li: perms[li % 2] for li in range(sh["layers"])}
    blocks = make_blocks(sh["layers"], sh["hidden"], sh["inter"], E, sh["top_k"], sh["family"],
                         sh["bits"], 64, sh["scale_dtype"], True, seed=52, device=dev)
    handle = attach(blocks, store, sh["capacity"], policy="lfuda", warm="auto", device=dev)
    h2d = _h2d_gbs(dev)
    res = {"capacity": sh["capacity"], "policy": "lfuda", "h2d_gbs_measured": h2d,
           "data": "8 experts N(0,0.02) quantised to 8-bit on the GPU, held once in pinned host "
                   "DRAM in two per-layer permutations that all 32 layers share (the copies "
                   "over PCIe are real); router N(0,0.02) + bias N(0,1) per layer"}
    # prefill: layer-major, token-wise: each layer's experts cross PCIe once per span
    handle.reset_stats()
    pf = _prefill_gemm(dev, blocks, sh["prefill"], 78, bf16_peak, bf16_kind,
                       layer_scope=handle.prefill_layer, warm=False)
    stp = handle.stats()
    pf["admit_gb"] = stp["admit_gb"]
    pf["pcie_gbs"] = stp["admit_gb"] / (pf["ms"] / 1e3)
    pf["pcie_frac"] = pf["pcie_gbs"] / h2d
    res["prefill"] = pf
    # decode sample: B=1 tokens through all layers, the routing read back per layer
    g = torch.Generator(device=dev)
    g.manual_seed(79)
    n_dec = 12
    xs = torch.randn(W + n_dec, 1, sh["hidden"], generator=g, device=dev).to(torch.bfloat16)
    for i in range(W):
        _normed_step(blocks, xs[i])
    handle.reset_stats()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(n_dec):
        _normed_step(blocks, xs[W + i])
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    st = handle.stats()
    res["decode"] = {"batch": 1, "tokens": n_dec, "tok_s": n_dec / (ms / 1e3),
                     "ms_per_token": ms / n_dec, "miss_rate": st["miss_rate"],
                     "admit_gb": st["admit_gb"], "pcie_gbs": st["admit_gb"] / (ms / 1e3),
                     "pcie_frac": st["admit_gb"] / (ms / 1e3) / h2d,
                     "stage_issued": st["stage_issued"], "stage_hits": st["stage_hits"],
                     "roofline": {"bound": "pcie", "achieved": st["admit_gb"] / (ms / 1e3),
                                  "peak": h2d, "unit": "GB/s",
                                  "frac": st["admit_gb"] / (ms / 1e3) / h2d,
                                  "note": "missed-expert bytes copied from pinned host over the "
                                          "decode time, against the measured pinned H2D rate"},
                     "note": f"{n_dec} decode tokens (a sample of the config's 512) after {W} "
                             f"warm-up tokens"}
    handle.close()
    del blocks, store, perms
    return res


# ------------------------------------------------------------------ CPU restatement
def cpu_decode_tokens(store, blocks_host, n_tokens: int, n_layers: int, threads: int, seed: int,
                      first_layer: int = 0):
    """Seconds per token of the numpy restatement over ``n_layers`` layers starting at
    ``first_layer`` (a bounded sample of the workload)."""
    from concurrent.futures import ThreadPoolExecutor
    from bigrig_b200.formats import make_spec, unpack_expert
    from oracle import affine, moe, router
    c = CFG
    spec = make_spec(c["hidden"], c["inter"], c["bits"], c["group_size"], c["scale_dtype"])
    rng = np.random.default_rng(seed)
    pool = ThreadPoolExecutor(max_workers=threads)

    def expert_w(li, e):
        a = unpack_expert(store.layers[li][e].numpy(), spec)
        return {p: affine.dequantize_f32(a[p]["weight"], a[p]["scales"], a[p]["biases"],
                                         c["group_size"], c["bits"], c["scale_dtype"])
                for p in moe.PROJ}

    t0 = time.perf_counter()
    for _ in range(n_tokens):
        h = affine.bf16_round(rng.standard_normal((1, c["hidden"])).astype(np.float32))
        for li in range(first_layer, first_layer + n_layers):
            gw, gb = blocks_host[li]
            lg = router.router_logits(h, gw, gb)
            idx, sc = router.topk(lg, c["top_k"], "softmax_topk", False)
            ws = list(pool.map(lambda e: expert_w(li, int(e)), idx[0]))
            y = np.concatenate([moe.expert_forward(h, w) for w in ws])[None]
            h = affine.bf16_round(h + moe.combine(y, sc))
    dt = time.perf_counter() - t0
    pool.shutdown()
    return dt / n_tokens


def _host_router(blocks):
    return [(b.gate_w.float().cpu().numpy(), b.gate_b.float().cpu().numpy()) for b in blocks]


def run_reference(args) -> None:
    """The reference arm: the CPU restatement of the same workload on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    c = CFG
    # weights are generated with the same seeded GPU quantiser when a GPU exists, else on CPU
    dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
    blocks, store = build_model(dev, seed=0)
    host = _host_router(blocks)
    # one step = one token through ONE MoE layer (a bounded 1/16 sample of a token)
    per_layer = []
    for i in range(args.warmup + args.steps):
        dt = cpu_decode_tokens(store, host, 1, 1, threads, seed=i, first_layer=i % c["layers"])
        if i >= args.warmup:
            per_layer.append(dt)
    sec_per_token = statistics.mean(per_layer) * c["layers"]
    v = 1.0 / sec_per_token
    line = {"metric": METRIC, "value": v, "unit": "tok/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(per_layer) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u4 codes, fp32 math",
            "data": "synthetic", "config": {k: CFG[k] for k in ("workload", "layers", "hidden", "inter", "experts", "top_k", "bits")},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": "each step: one token through one of the 16 MoE layers "
                                       "(numpy restatement, all experts resident in host RAM); "
                                       "tok/s = 1 / (16 x mean layer time)"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def ep_reference_check(dev, c: dict, stack, x: torch.Tensor, rank: int, world: int, dist) -> dict:
    """Layer by layer, every rank's token through the expert-parallel stack against the same
    layer input through one GPU holding every expert (on rank 0), under the expert parity
    bar |d| <= 2e-3 + 1e-2 |ref| per element.  All ranks run the EP layers (their
    collectives); rank 0 also builds the reference stack and returns the result."""
    ref_blocks = None
    if rank == 0:
        from bigrig_b200.stream import attach
        ref_blocks, store = build_model(dev, seed=0, layers=c["layers"])
        ref_handle = attach(ref_blocks, store, c["experts"], policy=c["policy"], warm="auto",
                            device=dev)
    # the other ranks wait here while rank 0 builds the reference (seconds): a peer-memory
    # layer's bounded waits must not start before every rank can answer them
    torch.cuda.synchronize(dev)
    dist.barrier()
    outside, worst, max_abs, n = 0, 0.0, 0.0, 0
    h = x
    for li, blk in enumerate(stack):
        # the layer's MoE output m, compared before the residual add: that add is one bf16
        # rounding of h + m, and where the two nearly cancel it turns a 1-ulp difference of
        # m (e.g. the grouped GEMM's fp16 weights against the one-token kernel's) into a
        # large relative one.  The next input, bf16(h + m), is what the fused residual form
        # gives bit for bit.
        m = blk(h)
        y = (h.float() + m.float()).to(torch.bfloat16)
        hs = [torch.empty_like(h) for _ in range(world)]
        ys = [torch.empty_like(m) for _ in range(world)]
        dist.all_gather(hs, h)
        dist.all_gather(ys, m)
        if rank == 0:
            for hi, yi in zip(hs, ys):
                ref = ref_blocks[li](hi).float()
                d = (yi.float() - ref).abs()
                allow = 2e-3 + 1e-2 * ref.abs()
                outside += int((d > allow).sum())
                worst = max(worst, float((d / allow).max()))
                max_abs = max(max_abs, float(d.max()))
                n += d.numel()
        h = y
    if rank != 0:
        return None
    ref_handle.close()
    return {"tokens": world, "layers": len(stack), "elements": n, "outside": outside,
            "max_abs": max_abs, "worst_vs_bar": worst, "ok": outside == 0,
            "note": "each rank's first timed token, layer by layer: the EP layer's MoE output "
                    "(before the residual add) vs the same input through one GPU with every "
                    "expert resident; bar 1e-2 rel / 2e-3 abs per element"}


# ------------------------------------------------------------------ the B200 arm
def _full_decode(dev, blocks, store, c: dict, steps: int = 256) -> dict:
    """BASELINE config 2 in full: embeddings, attention (MHA 16 x 128, KV cache), the 16 MoE
    layers over pools capped at 16/64 and refilled from pinned host, the LM head; a 2048-token
    random prompt (layer-major prefill), then ``steps`` greedy decode steps.  Attention and
    the LM head are bf16 cuBLAS/SDPA calls around the library's MoE layers."""
    from bigrig_b200.decoder import FAMILY_ATTN, Decoder
    from bigrig_b200.stream import attach
    handle = attach(blocks, store, c["capacity"], policy=c["policy"], warm="auto", device=dev)
    attn = FAMILY_ATTN["olmoe"]
    dec = Decoder(blocks, attn, c["prompt"] + steps, dev, seed=5)
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    prompt = torch.randint(0, attn.vocab, (c["prompt"],), generator=g, device=dev)
    # warm-up at the timed shapes: the whole prompt and a few steps (library set-up, cuBLAS
    # and attention kernels chosen for these shapes; the first pass costs ~1 s more)
    tok = dec.prefill(prompt, layer_scope=handle.prefill_layer)
    for _ in range(8):
        tok = dec.step(tok)
    dec.reset()
    handle.reset_stats()
    torch.cuda.synchronize(dev)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    e[0].record()
    tok = dec.prefill(prompt, layer_scope=handle.prefill_layer)
    e[1].record()
    for _ in range(steps):
        tok = dec.step(tok)
    e[2].record()
    torch.cuda.synchronize(dev)
    pf_ms, dc_ms = e[0].elapsed_time(e[1]), e[1].elapsed_time(e[2])
    st = handle.stats()
    out = {"workload": "olmoe-1b-7b-shaped full decode: 16 layers, MHA 16 x 128, vocab 50304, "
                       "pool 16/64 per layer refilled from pinned host; attention, embeddings "
                       "and LM head bf16 (random init)",
           "prompt": c["prompt"], "steps": steps,
           "prefill_tok_s": c["prompt"] / (pf_ms / 1e3), "prefill_ms": pf_ms,
           "decode_tok_s": steps / (dc_ms / 1e3), "decode_ms_per_token": dc_ms / steps,
           "miss_rate": st["miss_rate"], "admit_gb": st["admit_gb"]}
    return out                   # (the host store stays open: the CPU baseline reads it)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="decode only (for profiling)")
    ap.add_argument("--ep-slots", type=int, default=None,
                    help="expert-parallel runs: slots per layer per rank (default: the config's "
                         "capacity, at most the rank's experts)")
    ap.add_argument("--ep", default="peer", choices=["peer", "nccl"],
                    help="expert-parallel decode exchange: 'peer' stores rows into the other "
                         "ranks' buffers over NVLink inside the library's kernels (every local "
                         "expert resident); 'nccl' the all-to-all block over pools of --ep-slots")
    ap.add_argument("--configs", default="c3,c4,c5",
                    help="other BASELINE shapes measured at N=1 as extra keys (comma list of "
                         "c3, c4, c5, or 'none')")
    ap.add_argument("--path", default="auto", choices=["auto", "tiled", "split", "chain"],
                    help="expert-kernel path mode (bigrig_set_path); 'split' / 'tiled' pick the "
                         "one-token layer kernel (for profiler captures)")
    ap.add_argument("--layers", type=int, default=None,
                    help="MoE layers of the stack (default: the config's 16; fewer only to keep "
                         "a profiler capture small -- such a run is not a bench line)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
        return

    from bigrig_b200 import _lib, layered, ops
    from bigrig_b200.stream import attach

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.load(build_if_stale=False)
    _lib.set_path(args.path)
    c = dict(CFG)
    if args.layers is not None:
        c["layers"] = args.layers
    if world == 1:
        blocks, store = build_model(dev, seed=0, layers=c["layers"])
        handle = attach(blocks, store, c["capacity"], policy=c["policy"], warm="auto", device=dev)
        stack = blocks
    else:
        # expert parallel: this rank owns a contiguous block of every layer's experts, held
        # in a pool of min(capacity, E/N) slots; routed pairs travel by NCCL all-to-all
        from bigrig_b200.block import EPMoEBlock
        from bigrig_b200.ep import ExpertParallel
        from bigrig_b200.stream import ExpertPool, StreamHandle, StreamingSwitchGLU
        ep = ExpertParallel(c["experts"])
        lo, hi = ep.local_range()
        blocks, store = build_model(dev, seed=0, experts=range(lo, hi), layers=c["layers"])
        pools, mods = [], []
        slots = min(args.ep_slots or c["capacity"], hi - lo)
        if args.ep == "peer":
            slots = hi - lo                      # the peer path never reads routing back

        for b in blocks:
            pool = ExpertPool(b.layer, None, hi - lo, slots, b.spec,
                              policy=c["policy"], quant=b.quant, device=dev).build()
            pools.append(pool)
            mods.append(StreamingSwitchGLU(pool, store))
        handle = StreamHandle(blocks, pools, mods, store).warm("auto")
        for m in mods:
            m.refresh()
        stack = [EPMoEBlock(b, ep, m, padded=m._sync_free) for b, m in zip(blocks, mods)]
        if args.ep == "peer":
            # one-token decode layers exchange through peer memory; the prompt keeps the
            # NCCL all-to-all block
            from bigrig_b200.block import EPPeerBlock
            from bigrig_b200.ep import PeerBuffers
            peers = PeerBuffers(1, c["hidden"], c["top_k"], dev)
            stack = [EPPeerBlock(b, peers, m, lo, hi - lo, fallback=s)
                     for b, m, s in zip(blocks, mods, stack)]
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    W, K = args.warmup, args.steps
    tokens = torch.randn(W + K, 1, c["hidden"], generator=g, device=dev).to(torch.bfloat16)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    extras = {}
    # ---- prefill: the 2048-token prompt, layer-major, through the capped pools
    if not args.no_extras:
        prompt = torch.randn(c["prompt"], c["hidden"], generator=g, device=dev).to(torch.bfloat16)
        layers = [(lambda h, b=b: b(h, residual=h)) for b in stack]
        if world > 1:
            for b in stack:
                b.padded = False             # prompt chunks exchange exact row counts

        def capped_prefill(token_wise, name):
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push(name)
            e0.record()
            layered.prefill(layers, layered.chunks(prompt, c["prefill_chunk"]),
                            layer_scope=handle.prefill_layer, token_wise=token_wise)
            e1.record()
            torch.cuda.nvtx.range_pop()
            barrier()
            return max_over_ranks(e0.elapsed_time(e1))

        # a one-chunk pass first: library set-up (workspaces, tensor maps) outside the timing
        layered.prefill(layers, layered.chunks(prompt[:c["prefill_chunk"]], c["prefill_chunk"]),
                        layer_scope=handle.prefill_layer)
        pf_ms = capped_prefill(True, "prefill")
        pfc_ms = capped_prefill(False, "prefill_chunked")
        extras["prefill_tok_s"] = world * c["prompt"] / (pf_ms / 1e3)
        extras["prefill_chunked_tok_s"] = world * c["prompt"] / (pfc_ms / 1e3)
        extras["prefill_note"] = ("2048-token prompt, layer-major through the capped pools: "
                                  "prefill_tok_s token-wise (each layer once over the whole "
                                  "prompt, so every expert crosses PCIe once per layer), "
                                  "prefill_chunked_tok_s in the reference's chunks of 512 (a "
                                  "layer's experts cycle through the pool once per chunk); "
                                  "expert-sorted spans of <= capacity experts, tcgen05 grouped "
                                  "GEMM")
        if world > 1:
            for b in stack:
                b.padded = b.switch._sync_free
        handle.reset_stats()

    # ---- decode, capped pool: warm-up then K timed steps
    barrier()                                  # ranks meet before the first peer-memory layer
    for i in range(W):
        stack_step(stack, tokens[i])
    step, graph = stack_step, None
    if world > 1 and all(b.padded for b in stack):
        # every rank's pools hold all its experts: the whole step (router, the padded NCCL
        # all-to-alls, the expert kernels, the combines) is one CUDA graph per token
        for p in handle.pools:
            p.g2s_device()
            p.settle()
        xin = tokens[0].clone()
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                stack_step(stack, xin)
        torch.cuda.current_stream(dev).wait_stream(side)
        barrier()
        graph = torch.cuda.CUDAGraph()
        cap0 = _lib.launch_counts()
        with torch.cuda.graph(graph):
            yout = stack_step(stack, xin)
        cap1 = _lib.launch_counts()
        # the library counts a launch when it is issued: in a graph, once at capture, so a
        # replay runs the captured launches again
        graph_launches = {k: cap1[k] - cap0[k] for k in cap1}

        def step(_stack, x, _g=graph, _x=xin, _y=yout):
            _x.copy_(x)
            _g.replay()
            return _y
        for i in range(W):
            step(stack, tokens[i])
        barrier()
    handle.reset_stats()
    barrier()
    counts0 = _lib.launch_counts()
    _lib.timing_enable(["decode_split", "decode_layer"])
    clocks = Clocks(local)
    clocks.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("decode")
    t0.record()
    for i in range(K):
        step(stack, tokens[W + i])
    t1.record()
    torch.cuda.nvtx.range_pop()
    barrier()
    clk = clocks.stop()
    _lib.timing_enable([])
    counts1 = _lib.launch_counts()
    # the one-token layer kernel that ran: the split kernel where it fits, else the tiled one
    one_kernel = "decode_split"
    gu_ms, gu_n = _lib.timing_read("decode_split")
    t_ms, t_n = _lib.timing_read("decode_layer")
    if t_n > gu_n:
        one_kernel, gu_ms, gu_n = "decode_layer", t_ms, t_n
    ms = max_over_ranks(t0.elapsed_time(t1))
    value = world * K / (ms / 1e3)
    st = handle.stats()
    by_kernel = {k: counts1[k] - counts0[k] for k in counts1}
    if graph is not None:
        by_kernel = {k: by_kernel[k] + K * graph_launches[k] for k in by_kernel}
    launches = sum(by_kernel.values())

    # ---- e2e through the public API with host buffers: pinned in, result read back
    hbuf = tokens.cpu().pin_memory()
    outbuf = torch.empty(1, c["hidden"], dtype=torch.bfloat16).pin_memory()
    barrier()
    w0 = time.perf_counter()
    for i in range(K):
        x = hbuf[W + i].to(dev, non_blocking=True)
        y = step(stack, x)
        outbuf.copy_(y, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - w0)
    e2e = {"value": world * K / e2e_s, "unit": "tok/s",
           "h2d_bytes_per_step": c["hidden"] * 2, "d2h_bytes_per_step": c["hidden"] * 2,
           "note": "per step: token embedding copied from pinned host, 16 MoE layers, result "
                   "read back; misses copied from pinned host inside the step"}

    # ---- expert-parallel check: every rank's first timed token through the EP stack
    # against the same token through one GPU holding every expert (rank 0)
    ep_check = None
    peer_timeouts = None
    if world > 1 and args.ep == "peer":
        peer_timeouts = {"decode": peers.errors()}
    if world > 1:
        ep_check = ep_reference_check(dev, c, stack, tokens[W].clone(), rank, world, dist)
    if world > 1 and args.ep == "peer":
        peer_timeouts["check"] = peers.errors()
        t = torch.tensor([peer_timeouts["decode"], peer_timeouts["check"]], device=dev)
        dist.all_reduce(t)                 # every rank's count, summed
        peer_timeouts = {"decode": int(t[0]), "check": int(t[1]),
                         "note": "peer waits that ran out, all ranks: in the warm-up, timed and "
                                 "end-to-end decode, and in the expert-parallel check"}
        if ep_check is not None and peer_timeouts["check"]:
            ep_check["ok"] = False
    if graph is not None:
        del step, graph
        graph = None

    # ---- resident (sync-free) decode in one CUDA graph per token (single GPU)
    if not args.no_extras and world == 1:
        handle = None                    # its pools' slabs are freed once the blocks let go
        res = attach(blocks, store, c["experts"], policy=c["policy"], warm="auto", device=dev)
        ws = ops.default_workspace(dev)
        L0 = res.pools[0].layout
        ws.reserve(ops.workspace_bytes(1, c["top_k"], c["experts"], L0))
        for p in res.pools:
            p.g2s_device()
            p.settle()
        xin = tokens[0].clone()
        for i in range(3):
            stack_step(blocks, xin)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                stack_step(blocks, xin)
        torch.cuda.current_stream(dev).wait_stream(s)
        with torch.cuda.graph(graph):
            yout = stack_step(blocks, xin)
        for i in range(W):
            xin.copy_(tokens[i])
            graph.replay()
        barrier()
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("resident_decode")
        r0.record()
        for i in range(K):
            xin.copy_(tokens[W + i])
            graph.replay()
        r1.record()
        torch.cuda.nvtx.range_pop()
        barrier()
        rms = max_over_ranks(r0.elapsed_time(r1))
        res_tok_s = K / (rms / 1e3)
        layer_bytes = algorithmic_layer_bytes(1, c["top_k"])
        hbm_peak, _, peak_kind = _peaks()
        extras["resident_decode_tok_s"] = world * res_tok_s
        extras["moe_layer_hbm_gbs"] = layer_bytes * c["layers"] * res_tok_s / 1e9
        extras["moe_layer_hbm_frac"] = extras["moe_layer_hbm_gbs"] / hbm_peak
        extras["moe_layer_bytes"] = layer_bytes
        extras["resident_ms_per_token"] = rms / K
        del graph, yout

        # ---- resident prefill: the same prompt, layer-major, every expert in HBM -- the
        # tcgen05 grouped GEMM with nothing to fetch; its kernels timed with CUDA events.
        # Twice: in the reference's 512-token chunks, and token-wise (every chunk of a
        # layer in one call: the same rows and results, all of an expert's rows at once).
        res_layers = [(lambda h, b=b: b(h, residual=h)) for b in blocks]
        flops = 6.0 * c["prompt"] * c["top_k"] * c["hidden"] * c["inter"] * c["layers"]
        bf16_peak, bf16_kind = _bf16_sustained()

        def resident_prefill(token_wise):
            for _ in range(2):
                layered.prefill(res_layers, layered.chunks(prompt, c["prefill_chunk"]),
                                token_wise=token_wise)
            barrier()
            _lib.timing_enable(["gemm_gate_up", "gemm_down"])
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push("resident_prefill_tw" if token_wise else "resident_prefill")
            p0.record()
            layered.prefill(res_layers, layered.chunks(prompt, c["prefill_chunk"]),
                            token_wise=token_wise)
            p1.record()
            torch.cuda.nvtx.range_pop()
            barrier()
            _lib.timing_enable([])
            gu_ms_p, _ = _lib.timing_read("gemm_gate_up")
            dn_ms_p, _ = _lib.timing_read("gemm_down")
            rp_ms = max_over_ranks(p0.elapsed_time(p1))
            gemm_s = max_over_ranks(gu_ms_p + dn_ms_p) / 1e3
            achieved = flops / gemm_s / 1e12 if gemm_s > 0 else None
            return rp_ms, {
                "kernel": "grouped_gemm_kernel", "bound": "tensor",
                "achieved": achieved, "unit": "TFLOP/s", "peak": bf16_peak, "peak_kind": bf16_kind,
                "frac": achieved / bf16_peak if achieved else None,
                "flops": flops, "gemm_ms": gemm_s * 1e3, "prefill_ms": rp_ms,
                "gate_up_ms": gu_ms_p, "down_ms": dn_ms_p,
                "note": "6 x prompt x top_k x hidden x inter x layers over the gate/up + down "
                        "GEMM launch time of a 2048-token layer-major prefill with every expert "
                        "resident, " + ("token-wise (one call per layer)" if token_wise else
                                        f"in chunks of {c['prefill_chunk']}")}

        rp_ms, extras["prefill_gemm"] = resident_prefill(False)
        extras["resident_prefill_tok_s"] = world * c["prompt"] / (rp_ms / 1e3)
        rp_tw, extras["prefill_gemm_token_wise"] = resident_prefill(True)
        extras["resident_prefill_token_wise_tok_s"] = world * c["prompt"] / (rp_tw / 1e3)

    # ---- config 2 in full: attention, KV cache and LM head around the capped MoE stack
    if not args.no_extras and world == 1 and c["layers"] == CFG["layers"]:
        extras["full_decode"] = _full_decode(dev, blocks, store, c)

    # ---- the other named shapes, one GPU
    if not args.no_extras and world == 1 and args.configs != "none":
        hbm_peak, _, hbm_kind = _peaks()
        burst = _peaks()[1]
        for key in [k.strip() for k in args.configs.split(",") if k.strip()]:
            extras[key] = bench_shape(dev, key, W, hbm_peak, hbm_kind, burst, "measured burst")

    # ---- CPU restatement on rank 0 at N=1 (bounded sample)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        per_tok = cpu_decode_tokens(store, _host_router(blocks), 2, c["layers"], threads, seed=7)
        cpu = {"value": 1.0 / per_tok, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": "2 decode tokens through all 16 MoE layers, numpy restatement "
                         "(dequantise the 8 routed experts per layer, fp32 math)"}

    hbm_peak, _, peak_kind = _peaks()
    gu_avg_ms = gu_ms / max(1, gu_n)
    gu_bytes = algorithmic_layer_bytes(1, c["top_k"])
    achieved = gu_bytes / (gu_avg_ms / 1e3) / 1e9 if gu_n else None
    traffic = _traffic().get(f"{one_kernel}_kernel")
    if "moe_layer_hbm_gbs" in extras:
        # the persistent one-token layer kernel of the resident decode: algorithmic bytes of
        # a layer over the graph's time per layer (which includes the launch gap)
        extras["resident_roofline"] = {
            "kernel": f"{one_kernel}_kernel", "bound": "hbm",
            "achieved": extras["moe_layer_hbm_gbs"], "peak": hbm_peak, "unit": "GB/s",
            "frac": extras["moe_layer_hbm_gbs"] / hbm_peak, "peak_kind": peak_kind,
            "traffic": _traffic().get(f"{one_kernel}_kernel"),
            "bytes_per_launch": extras["moe_layer_bytes"],
            "avg_launch_ms": extras["resident_ms_per_token"] / c["layers"]}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 activations, u4 affine codes, fp32 accumulate",
            "data": "synthetic: N(0,1) bf16 token embeddings, N(0,0.02) experts quantised to "
                    "MLX affine 4-bit g64, router bias N(0,1); random init",
            "config": {**{k: c[k] for k in ("workload", "layers", "hidden", "inter", "experts",
                                            "top_k", "bits", "group_size", "capacity", "policy")},
                       "global_batch": world,
                       "parallelism": "single GPU" if world == 1 else
                       f"ep{world}: {c['experts'] // world} experts per rank per layer, all "
                       f"resident; decode rows exchanged by stores into peer buffers over "
                       f"NVLink (gather, expert kernels, scatter, combine)" if args.ep == "peer"
                       else f"ep{world}: {c['experts'] // world} experts per rank per layer, "
                       f"pool {min(args.ep_slots or c['capacity'], c['experts'] // world)} "
                       f"slots, NCCL all-to-all",
                       "l2": "decode reads 28 MB of experts per layer, 453 MB per token; no flush"},
            "e2e": e2e,
            "gpu_launches": launches,
            "launches_by_kernel": by_kernel,
            "roofline": {"kernel": f"{one_kernel}_kernel" if gu_n else
                         "none: no one-token layer kernel ran (expert-parallel decode runs the "
                         "GEMV chain or grouped GEMM over the pairs routed to the rank's "
                         "experts)",
                         "bound": "hbm", "achieved": achieved,
                         "peak": hbm_peak, "unit": "GB/s",
                         "frac": (achieved / hbm_peak) if achieved else None,
                         "peak_kind": peak_kind, "traffic": traffic if gu_n else None,
                         "bytes_per_launch": gu_bytes, "avg_launch_ms": gu_avg_ms,
                         "timed_launches": gu_n},
            "pool": {"miss_rate": st["miss_rate"], "hits": st["hits"], "misses": st["misses"],
                     "admit_gb": st["admit_gb"], "sync_seconds": st["sync_seconds"],
                     "stage_issued": st.get("stage_issued"), "stage_hits": st.get("stage_hits")},
            "clocks": clk,
            "cpu_baseline": cpu,
            **({"ep_check": ep_check, "ep_graph": bool(world > 1 and all(b.padded for b in stack))}
               if world > 1 else {}),
            **({"peer_wait_timeouts": peer_timeouts} if peer_timeouts is not None else {}),
            **extras,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        if world > 1 and args.ep == "peer":
            peers.close()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
