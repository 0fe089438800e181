"""Torch-tensor wrappers over the C-ABI entry points (include/bigrig_b200.h).

Torch owns every allocation (device tensors, the per-device workspace); the
library only reads and writes what it is handed, on the caller's current CUDA
stream.  Every function here requires CUDA tensors and raises otherwise: there
is no CPU implementation of the hot path in the product.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _lib
from .formats import Layout

_MODES = {"softmax_topk": _lib.SOFTMAX_TOPK, "topk_softmax": _lib.TOPK_SOFTMAX}
_HALF = {"float16": torch.float16, "bfloat16": torch.bfloat16}


def _vp(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _require_cuda(name: str, t: torch.Tensor, dtype=None) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor: the MoE hot path runs only on the "
                           f"sm_100a kernels of libbigrig_b200.so (no CPU fallback)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


_raw_stream = torch._C._cuda_getCurrentRawStream


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    """The caller's current CUDA stream on ``t``'s device (the raw handle: a decode step makes
    several of these calls per layer, and building a torch Stream object for each shows)."""
    return ctypes.c_void_p(_raw_stream(t.get_device()))


_layout_cache: dict = {}
_layout_by_id: dict = {}
_stream_objs: dict = {}


def current_stream(device_index: int) -> torch.cuda.Stream:
    """torch's current stream on a device, the object looked up by its raw handle (building
    a Stream object per call costs several microseconds; a decode step needs a few per layer)."""
    raw = _raw_stream(device_index)
    s = _stream_objs.get((device_index, raw))
    if s is None:
        s = _stream_objs[(device_index, raw)] = torch.cuda.current_stream(device_index)
    return s


def c_layout(L: Layout) -> _lib.ExpertLayout:
    """The ctypes struct of a Layout (cached; checked once by the library)."""
    hit = _layout_by_id.get(id(L))
    if hit is not None and hit[0] is L:
        return hit[1]
    c = _layout_cache.get(L)
    if c is None:
        c = _lib.ExpertLayout()
        c.hidden, c.inter, c.bits, c.group_size = L.hidden, L.inter, L.bits, L.group_size
        c.scale_dtype, c.flags = L.scale_code, L.flags
        c.bytes_per_expert, c.slot_stride = L.bytes_per_expert, L.slot_stride
        for i in range(3):
            c.weight_off[i], c.scales_off[i], c.biases_off[i] = (L.weight_off[i], L.scales_off[i],
                                                                 L.biases_off[i])
            c.bias_off[i] = L.bias_off[i]
        _lib.check(_lib.load().bigrig_check_layout(ctypes.byref(c)), "layout")
        _layout_cache[L] = c
    _layout_by_id[id(L)] = (L, c)
    return c


class Workspace:
    """Zero-initialised device scratch for MoE calls, grown on demand.

    Size it up front (``reserve``) for the largest call before capturing a CUDA
    graph: growing allocates, which a capture must not do.
    """

    def __init__(self, device):
        self.device = torch.device(device)
        self.buf = torch.zeros(0, dtype=torch.uint8, device=self.device)

    def reserve(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            self.buf = torch.zeros(int(nbytes), dtype=torch.uint8, device=self.device)
        return self.buf

    def errors(self) -> int:
        """Read and clear the device error word (missing slots, ids out of range)."""
        out = ctypes.c_int32(0)
        _lib.check(_lib.load().bigrig_workspace_errors(
            _vp(self.buf), ctypes.byref(out), _stream(self.buf)), "workspace_errors")
        return int(out.value)


_ws_lock = threading.Lock()
_workspaces: dict = {}


def default_workspace(device) -> Workspace:
    d = torch.device(device)
    key = (d.type, d.index if d.index is not None else torch.cuda.current_device())
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None:
            ws = _workspaces[key] = Workspace(torch.device("cuda", key[1]))
        return ws


_ws_bytes: dict = {}


def workspace_bytes(T: int, k: int, n_experts: int, layout: Layout) -> int:
    key = (T, k, n_experts, layout)
    n = _ws_bytes.get(key)
    if n is None:
        n = _ws_bytes[key] = int(_lib.load().bigrig_moe_workspace_bytes(
            T, k, n_experts, ctypes.byref(c_layout(layout))))
    return n


# ------------------------------------------------------------------ entry points
def dequant(slab: torch.Tensor, layout: Layout, slot: int, proj: int) -> torch.Tensor:
    """Dequantised projection ``proj`` (0 gate, 1 up, 2 down) of slot ``slot``, in the scale dtype."""
    _require_cuda("slab", slab, torch.uint8)
    if not 0 <= slot < slab.shape[0]:
        raise ValueError(f"slot {slot} outside the slab's {slab.shape[0]} slots")
    rows, cols = (layout.hidden, layout.inter) if proj == 2 else (layout.inter, layout.hidden)
    out = torch.empty(rows, cols, dtype=_HALF[layout.scale_dtype], device=slab.device)
    _lib.check(_lib.load().bigrig_dequant(_vp(slab), ctypes.byref(c_layout(layout)), slot, proj,
                                          _vp(out), _stream(slab)), "dequant")
    return out


def router_logits(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 logits[T, E] = x[T, H] . w[E, H]^T (+ bias[E]); x and w bf16.  ``out``, when
    given, is a contiguous fp32 tensor of T*E elements."""
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("w", w, torch.bfloat16)
    if bias is not None:
        _require_cuda("bias", bias, torch.float32)
    T, H = x.shape
    E = w.shape[0]
    if out is None:
        out = torch.empty(T, E, dtype=torch.float32, device=x.device)
    else:
        _require_cuda("out", out, torch.float32)
        if out.numel() != T * E:
            raise ValueError(f"out holds {out.numel()} logits, the call makes {T * E}")
    _lib.check(_lib.load().bigrig_router_logits(_vp(x), _vp(w), _vp(bias), _vp(out), T, H, E,
                                                _stream(x)), "router_logits")
    return out


def router_topk(logits: torch.Tensor, k: int, mode: str = "softmax_topk", norm_topk: bool = False,
                indices: torch.Tensor | None = None, scores: torch.Tensor | None = None):
    """(indices int32 [T, k] in rank order, scores fp32 [T, k])."""
    _require_cuda("logits", logits)
    if logits.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"logits must be float32 or bfloat16, got {logits.dtype}")
    if mode not in _MODES:
        raise ValueError(f"mode must be one of {tuple(_MODES)}, got {mode!r}")
    T, E = logits.shape
    if indices is None:
        indices = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    if scores is None:
        scores = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    dt = _lib.F32 if logits.dtype == torch.float32 else _lib.BF16
    _lib.check(_lib.load().bigrig_router_topk(_vp(logits), dt, T, E, k, _MODES[mode], int(norm_topk),
                                              _vp(indices), _vp(scores), _stream(logits)),
               "router_topk")
    return indices, scores


def moe_permute(indices: torch.Tensor, n_experts: int) -> dict:
    """Stable expert-sorted permutation of indices[T, k]; see bigrig_moe_permute."""
    _require_cuda("indices", indices, torch.int32)
    T, k = indices.shape
    dev = indices.device
    P = T * k
    out = {"order": torch.empty(P, dtype=torch.int32, device=dev),
           "inv": torch.empty(P, dtype=torch.int32, device=dev),
           "offsets": torch.empty(n_experts + 1, dtype=torch.int32, device=dev),
           "seg_expert": torch.full((n_experts,), -1, dtype=torch.int32, device=dev),
           "seg_start": torch.full((n_experts + 1,), -1, dtype=torch.int32, device=dev),
           "num_seg": torch.zeros(1, dtype=torch.int32, device=dev),
           "err": torch.zeros(1, dtype=torch.int32, device=dev)}
    _lib.check(_lib.load().bigrig_moe_permute(
        _vp(indices), T, k, n_experts, _vp(out["order"]), _vp(out["inv"]), _vp(out["offsets"]),
        _vp(out["seg_expert"]), _vp(out["seg_start"]), _vp(out["num_seg"]), _vp(out["err"]),
        _stream(indices)), "moe_permute")
    return out


def switch_glu(x: torch.Tensor, indices: torch.Tensor, slab: torch.Tensor, layout: Layout,
               n_experts: int, g2s: torch.Tensor | None = None, out: torch.Tensor | None = None,
               workspace: Workspace | None = None) -> torch.Tensor:
    """Unreduced expert outputs y[T, k, H] (bf16) of x[T, H] (bf16) routed by indices[T, k]."""
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("indices", indices, torch.int32)
    _require_cuda("slab", slab, torch.uint8)
    if g2s is not None:
        _require_cuda("g2s", g2s, torch.int32)
    T, k = indices.shape
    if x.shape != (T, layout.hidden):
        raise ValueError(f"x is {tuple(x.shape)}, expected ({T}, {layout.hidden})")
    if out is None:
        out = torch.empty(T, k, layout.hidden, dtype=torch.bfloat16, device=x.device)
    ws = workspace or default_workspace(x.device)
    need = workspace_bytes(T, k, n_experts, layout)
    buf = ws.reserve(need)
    _lib.check(_lib.load().bigrig_switch_glu(
        _vp(x), _vp(indices), T, k, n_experts, _vp(g2s), _vp(slab), ctypes.byref(c_layout(layout)),
        _vp(out), _vp(buf), buf.numel(), _stream(x)), "switch_glu")
    return out


def combine(y: torch.Tensor, scores: torch.Tensor, out: torch.Tensor | None = None,
            residual: torch.Tensor | None = None) -> torch.Tensor:
    """out[T, H] = sum_j scores[t, j] * y[t, j, :] (bf16 out, fp32 accumulation),
    plus ``residual`` when given (then out = bf16(residual + bf16(sum)))."""
    _require_cuda("y", y, torch.bfloat16)
    _require_cuda("scores", scores, torch.float32)
    T, k, H = y.shape
    if out is None:
        out = torch.empty(T, H, dtype=torch.bfloat16, device=y.device)
    if residual is None:
        _lib.check(_lib.load().bigrig_combine(_vp(y), _vp(scores), T, k, H, _vp(out), _stream(y)),
                   "combine")
    else:
        _require_cuda("residual", residual, torch.bfloat16)
        # the residual form is the combine kernel's second mode, reached through moe_layer's
        # fallback; here it is one elementwise step on top of the plain combine
        plain = torch.empty_like(out)
        _lib.check(_lib.load().bigrig_combine(_vp(y), _vp(scores), T, k, H, _vp(plain),
                                              _stream(y)), "combine")
        torch.add(residual, plain, out=out)
    return out


def moe_forward(x: torch.Tensor, logits: torch.Tensor, top_k: int, slab: torch.Tensor,
                layout: Layout, n_experts: int, mode: str = "softmax_topk",
                norm_topk: bool = False, g2s: torch.Tensor | None = None,
                out: torch.Tensor | None = None, indices: torch.Tensor | None = None,
                scores: torch.Tensor | None = None, workspace: Workspace | None = None):
    """Combined MoE output out[T, H] from router logits; returns (out, indices, scores)."""
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("logits", logits)
    _require_cuda("slab", slab, torch.uint8)
    if mode not in _MODES:
        raise ValueError(f"mode must be one of {tuple(_MODES)}, got {mode!r}")
    T = x.shape[0]
    dev = x.device
    if out is None:
        out = torch.empty(T, layout.hidden, dtype=torch.bfloat16, device=dev)
    if indices is None:
        indices = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    if scores is None:
        scores = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    dt = _lib.F32 if logits.dtype == torch.float32 else _lib.BF16
    ws = workspace or default_workspace(dev)
    buf = ws.reserve(workspace_bytes(T, top_k, n_experts, layout))
    _lib.check(_lib.load().bigrig_moe_forward(
        _vp(x), _vp(logits), dt, T, n_experts, top_k, _MODES[mode], int(norm_topk), _vp(g2s),
        _vp(slab), ctypes.byref(c_layout(layout)), _vp(out), _vp(indices), _vp(scores), _vp(buf),
        buf.numel(), _stream(x)), "moe_forward")
    return out, indices, scores


def moe_layer(x: torch.Tensor, gate_w: torch.Tensor, gate_b: torch.Tensor | None, top_k: int,
              slab: torch.Tensor, layout: Layout, n_experts: int, mode: str = "softmax_topk",
              norm_topk: bool = False, g2s: torch.Tensor | None = None,
              residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
              indices: torch.Tensor | None = None, scores: torch.Tensor | None = None,
              workspace: Workspace | None = None):
    """The MoE block from hidden states: router logits, top-k + softmax, experts, combine,
    plus ``residual`` when given.  Returns (out, indices, scores)."""
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("gate_w", gate_w, torch.bfloat16)
    _require_cuda("slab", slab, torch.uint8)
    if gate_b is not None:
        _require_cuda("gate_b", gate_b, torch.float32)
    if residual is not None:
        _require_cuda("residual", residual, torch.bfloat16)
    if mode not in _MODES:
        raise ValueError(f"mode must be one of {tuple(_MODES)}, got {mode!r}")
    T = x.shape[0]
    dev = x.device
    if out is None:
        out = torch.empty(T, layout.hidden, dtype=torch.bfloat16, device=dev)
    if indices is None:
        indices = torch.empty(T, top_k, dtype=torch.int32, device=dev)
    if scores is None:
        scores = torch.empty(T, top_k, dtype=torch.float32, device=dev)
    ws = workspace or default_workspace(dev)
    buf = ws.reserve(workspace_bytes(T, top_k, n_experts, layout))
    _lib.check(_lib.load().bigrig_moe_layer(
        _vp(x), _vp(gate_w), _vp(gate_b), T, n_experts, top_k, _MODES[mode], int(norm_topk),
        _vp(g2s), _vp(slab), ctypes.byref(c_layout(layout)), _vp(residual), _vp(out),
        _vp(indices), _vp(scores), _vp(buf), buf.numel(), _stream(x)), "moe_layer")
    return out, indices, scores


def moe_layer_routed(x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor,
                     slab: torch.Tensor, layout: Layout, n_experts: int,
                     g2s: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                     out: torch.Tensor | None = None,
                     workspace: Workspace | None = None) -> torch.Tensor:
    """The MoE block from routing already computed: x bf16 [T, H], indices int32 [T, k] and
    scores fp32 [T, k] on the device -> out bf16 [T, H] = residual + sum_j score * y."""
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("indices", indices, torch.int32)
    _require_cuda("scores", scores, torch.float32)
    _require_cuda("slab", slab, torch.uint8)
    if g2s is not None:
        _require_cuda("g2s", g2s, torch.int32)
    if residual is not None:
        _require_cuda("residual", residual, torch.bfloat16)
    T, k = indices.shape
    if tuple(scores.shape) != (T, k):
        raise ValueError(f"scores must be [{T}, {k}], got {tuple(scores.shape)}")
    x = x.contiguous()
    if out is None:
        out = torch.empty(T, layout.hidden, dtype=torch.bfloat16, device=x.device)
    ws = workspace or default_workspace(x.device)
    buf = ws.reserve(workspace_bytes(T, k, n_experts, layout))
    _lib.check(_lib.load().bigrig_moe_layer_routed(
        _vp(x), _vp(indices), _vp(scores), T, n_experts, k, _vp(g2s), _vp(slab),
        ctypes.byref(c_layout(layout)), _vp(residual), _vp(out), _vp(buf), buf.numel(),
        _stream(x)), "moe_layer_routed")
    return out


def switch_glu_noalloc(x: torch.Tensor, indices: torch.Tensor, slab: torch.Tensor, layout: Layout,
                       n_experts: int, g2s: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """switch_glu for callers that cannot allocate device memory when they call.

    The library keeps this call's scratch in a fixed 4 MiB device array (per GPU, for the
    life of the process) instead of a workspace; ``out`` must be preallocated for the call
    itself to allocate nothing.  Calls needing more scratch raise ValueError.  Concurrent
    calls on different streams share that array and must be serialised by the caller.
    """
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("indices", indices, torch.int32)
    _require_cuda("slab", slab, torch.uint8)
    if g2s is not None:
        _require_cuda("g2s", g2s, torch.int32)
    T, k = indices.shape
    if out is None:
        out = torch.empty(T, k, layout.hidden, dtype=torch.bfloat16, device=x.device)
    _lib.check(_lib.load().bigrig_switch_glu_noalloc(
        _vp(x), _vp(indices), T, k, n_experts, _vp(g2s), _vp(slab), ctypes.byref(c_layout(layout)),
        _vp(out), _stream(x)), "switch_glu_noalloc")
    return out


def peer_workspace_bytes(peers, n_experts: int, n_local: int, layout: Layout) -> int:
    """Scratch of one ``peer_layer`` call of this group."""
    n = _lib.load().bigrig_peer_workspace_bytes(ctypes.byref(peers.c), n_experts, n_local,
                                                ctypes.byref(c_layout(layout)))
    if n == 0:
        raise ValueError("peer_workspace_bytes: invalid group or layer")
    return int(n)


def peer_layer(peers, x: torch.Tensor, gate_w: torch.Tensor, gate_b: torch.Tensor | None,
               n_experts: int, first: int, n_local: int, slab: torch.Tensor, layout: Layout,
               mode: str = "softmax_topk", norm_topk: bool = False,
               g2s: torch.Tensor | None = None, residual: torch.Tensor | None = None,
               out: torch.Tensor | None = None, workspace: Workspace | None = None) -> torch.Tensor:
    """One expert-parallel MoE layer over the peer buffers of ``peers`` (ep.PeerBuffers):
    x bf16 [tokens, H] are this rank's rows; every rank calls it with its own rows and the
    same router; this rank's experts are [first, first + n_local) held in ``slab``
    (``g2s`` maps them, numbered from 0, to slots).  Returns out [tokens, H] =
    residual + sum_j score * y for this rank's rows."""
    _require_cuda("x", x, torch.bfloat16)
    _require_cuda("gate_w", gate_w, torch.bfloat16)
    _require_cuda("slab", slab, torch.uint8)
    if gate_b is not None:
        _require_cuda("gate_b", gate_b, torch.float32)
    if residual is not None:
        _require_cuda("residual", residual, torch.bfloat16)
    if mode not in _MODES:
        raise ValueError(f"mode must be one of {tuple(_MODES)}, got {mode!r}")
    if tuple(x.shape) != (peers.tokens, peers.hidden):
        raise ValueError(f"x must be [{peers.tokens}, {peers.hidden}], got {tuple(x.shape)}")
    x = x.contiguous()
    if out is None:
        out = torch.empty(peers.tokens, layout.hidden, dtype=torch.bfloat16, device=x.device)
    ws = workspace or default_workspace(x.device)
    buf = ws.reserve(peer_workspace_bytes(peers, n_experts, n_local, layout))
    _lib.check(_lib.load().bigrig_peer_layer(
        ctypes.byref(peers.c), _vp(x), _vp(gate_w), _vp(gate_b), n_experts, _MODES[mode],
        int(norm_topk), first, n_local, _vp(g2s), _vp(slab), ctypes.byref(c_layout(layout)),
        _vp(residual), _vp(out), _vp(buf), buf.numel(), _stream(x)), "peer_layer")
    return out
