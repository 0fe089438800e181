"""The bounded expert pool on HBM and the SwitchGLU-style layer that computes over it.

Drop-in for bigrig_engine/stream.py's ExpertPool (stream.py:454-810),
StreamingSwitchGLU (stream.py:814-1631), attach/StreamHandle (stream.py:1842-2200).

B200 design:

* A layer's pool is one HBM slab ``[capacity, slot_stride]`` (uint8).  A slot
  holds one expert's packed bytes exactly as they lie in the blob, so the sm_100a
  kernels read codes, scales and biases in place and an admission is one copy.
* Misses are copied from pinned host DRAM (fetch.HostExpertStore) with
  ``cudaMemcpyAsync`` on the pool's side stream.  An event orders each layer's
  copies before its kernels; a second event orders a slot's overwrite after the
  last kernel that read it, so copy and compute overlap without a race.
* Residency decisions are the reference's, step for step: ``touch`` in
  ascending expert id with each expert's best router rank, staged admissions
  first, then cold ones in ``need`` order, victims from the policy with
  ``exclude=protect`` (or least-recently-admitted when the policy cannot name a
  legal one), free slots popped from the end of the free list.  The golden replay
  in tests/golden/ensure_golden.npz pins the slot ids and tables.
* A pool holding every expert (``full``) is sync-free: expert ids become slots
  on the device (``g2s_device``), nothing is read back to the host.

The layer returns per-(token, k) outputs unreduced, ``y[..., k, H]``; the MoE
block applies the router weights (stream.py:1523-1525).
"""
from __future__ import annotations

import contextlib
import ctypes
import json
import os
import time

import numpy as np
import torch

from . import _lib, ops
from .formats import MLP_PROJECTIONS, PROJECTIONS, bytes_per_expert, layout_from_spec
from .residency import SlotTable

# Most experts a layer copies to the GPU on the previous layer's prediction -- the router's
# top-k, as in the reference (stream.py:1723-1726).
STAGE_MAX = 8
# Whether a layer stages the next layer's predicted experts (pinned host -> HBM staging
# buffers, on the copy stream, behind its own misses) while its experts compute.  The
# reference keeps this off (stream.py:1731-1758): on unified memory the staging copy
# contended with the expert reads.  On a discrete GPU it runs over PCIe beside the HBM-bound
# compute; the next layer's own router, evaluated in the same two launches as this layer's
# routing, names about 92 % of the next layer's misses (95 % of what it stages is used, on
# the synthetic OLMoE stack), and the copies leave the critical path: capped decode 202 ->
# 213 tok/s.  On by default; BIGRIG_STAGE=0 turns it off.
STAGING = os.environ.get("BIGRIG_STAGE", "1") != "0"


def projections_of(spec: dict) -> tuple:
    """The projections this layer's experts carry, in packed byte order (stream.py:66-68)."""
    return tuple(spec)


def is_gated(projections) -> bool:
    return "gate_proj" in tuple(projections)


def _call(rc: int, what: str) -> None:
    """A library status code: raise on anything but BIGRIG_OK."""
    if rc:
        _lib.check(rc, what)


def _as_u8(blob) -> torch.Tensor:
    """Host bytes of any kind (bytes, memoryview, numpy, tensor) as a flat uint8 tensor."""
    if isinstance(blob, torch.Tensor):
        return blob.reshape(-1).view(torch.uint8) if blob.dtype != torch.uint8 else blob.reshape(-1)
    if isinstance(blob, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(blob).view(np.uint8).reshape(-1))
    return torch.from_numpy(np.frombuffer(blob, dtype=np.uint8).copy())


class ExpertPool(SlotTable):
    """C slots of one layer's experts in HBM; the residency tables come from ``SlotTable``.

    Same constructor, methods, counters and exceptions as the reference
    (stream.py:501-810).  ``views`` is accepted for interface compatibility: on a
    discrete GPU there are no page-cache views, every resident expert is a slot.
    """

    def __init__(self, layer: int, sg, n_experts: int, capacity: int, spec: dict,
                 policy: str = "lfuda", quant: dict | None = None, views: bool = False,
                 device=None, copy_stream: torch.cuda.Stream | None = None):
        super().__init__(layer, n_experts, capacity, policy)
        self.sg, self.spec, self.views = sg, spec, bool(views)
        self.projections = projections_of(spec)
        self.gated = is_gated(self.projections)
        self.spec_quant = dict(quant or {"bits": 4, "group_size": 64, "mode": "affine"})
        self.layout = layout_from_spec(spec, self.spec_quant)
        self._bpe = bytes_per_expert(spec)
        if device is None:
            device = (torch.device("cuda", torch.cuda.current_device())
                      if torch.cuda.is_available() else "cpu")
        self.device = torch.device(device)
        # the HBM side: the slab, its copy stream and the two events ordering copies and reads
        self.slab: torch.Tensor | None = None
        self._built = False
        self._copy_stream = copy_stream
        self._copies_done = None     # event: this pool's queued admissions have landed
        self._reads_done = None      # event: the last kernel that read the slab has finished
        self._batch = None           # slot writes collected by ensure(), issued in one call
        self._g2s_dev = None
        self._widen = self.layout.source_bits == 3   # 3-bit codes widened into 4-bit slots
        self._landing = None
        self.admit_seconds = 0.0
        self.admit_bytes = 0
        # staging: experts the previous layer predicted for this one, copied ahead of need
        self.stage_pred = None
        self.stage = {}              # expert id -> its bytes in a staging buffer
        self._stage_buf = None       # [STAGE_MAX, bytes_per_expert] in HBM, made on first use
        self.stage_issued = self.stage_hits = self.zero_copy_admits = 0

    @property
    def stage_rows(self) -> int:
        """Staging buffers of this pool: at most STAGE_MAX, and never more than the pool's
        capacity (a step cannot admit more than that)."""
        return min(STAGE_MAX, self.capacity)

    def adopt(self, slab: torch.Tensor) -> "ExpertPool":
        """Make every expert resident from a device slab that already holds them, expert e in
        row e (``[n_experts, slot_stride]`` uint8 on this pool's device): a whole layer loaded
        straight into HBM, with no host copy.  Only for a pool whose capacity is the expert
        count; the slab becomes the pool's."""
        if self.capacity != self.n_experts:
            raise ValueError(f"layer {self.layer}: adopt() fills every slot, so the capacity "
                             f"must be {self.n_experts}, got {self.capacity}")
        want = (self.n_experts, self.layout.slot_stride)
        if tuple(slab.shape) != want or slab.dtype != torch.uint8 or slab.device != self.device:
            raise ValueError(f"layer {self.layer}: adopt() needs uint8 {want} on {self.device}, "
                             f"got {slab.dtype} {tuple(slab.shape)} on {slab.device}")
        self.slab = slab
        self._built = True
        if self.device.type == "cuda" and self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device=self.device)
        self._free = []
        for e in range(self.n_experts):
            self._miss_rank = {e: 0}
            self._placed(e, e)
        return self

    # -- construction -------------------------------------------------------
    @property
    def bytes_per_expert(self) -> int:
        return self._bpe

    def build(self):
        """Allocate the HBM slab.  The model's (E, ...) expert tensors, if ``sg`` holds
        any, are dropped first so both never coexist (stream.py:570-597)."""
        if self.sg is not None:
            for proj in self.projections:
                mod = getattr(self.sg, proj, None)
                if isinstance(mod, dict):
                    for comp in list(self.spec[proj]):
                        mod.pop(comp, None)
        self.slab = torch.empty((self.capacity, self.layout.slot_stride), dtype=torch.uint8,
                                device=self.device)
        if self.device.type == "cuda" and self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device=self.device)
        self._built = True
        return self

    def nbytes(self) -> int:
        return 0 if self.slab is None else self.slab.numel()

    def expert_arrays(self, e: int) -> torch.Tensor:
        """Resident expert e's packed bytes (a view of its slot).  KeyError if absent."""
        slot = int(self.g2s[int(e)])
        if slot < 0:
            raise KeyError(e)
        return self.slab[slot, :self.layout.bytes_per_expert]

    views_of = expert_arrays

    def admit(self, e: int, blob, protect=()) -> int:
        """Copy expert e's packed bytes into a slot and return the slot (stream.py:692-705)."""
        t0 = time.perf_counter()
        if not self._built:
            raise RuntimeError("admit() before build(): the pool has no slab yet")
        src = _as_u8(blob)
        if src.numel() != self.bytes_per_expert:
            raise ValueError(
                f"layer {self.layer} expert {e}: got {src.numel()} bytes, the layout needs "
                f"{self.bytes_per_expert}; a short or long region would leave the slot holding "
                f"parts of two experts, so nothing is written")
        return self.admit_arrays(e, src, protect=protect, _t0=t0)

    def build_arrays(self, e: int, blob) -> torch.Tensor:
        """One expert's bytes staged on the device, ready for admit_arrays (stream.py:707-755).

        A staged expert is bit-for-bit what a direct admit writes: the same bytes."""
        src = _as_u8(blob)
        if src.numel() != self.bytes_per_expert:
            raise ValueError(f"expert {e}: manifest accounts for {self.bytes_per_expert} bytes "
                             f"but the region is {src.numel()}.")
        if self.device.type != "cuda":
            return src.clone()
        with torch.cuda.stream(self._copy_stream):
            return src.to(self.device, non_blocking=src.is_pinned())

    def stage_experts(self, items) -> int:
        """stage_expert for several (expert, blob) pairs with one library call issuing the
        copies; returns how many were staged."""
        picked = []
        for e, blob in items:
            e = int(e)
            if self.g2s[e] >= 0 or e in self.stage or len(self.stage) + len(picked) >= self.stage_rows:
                continue
            if any(e == p for p, _ in picked):
                continue
            src = _as_u8(blob)
            if src.numel() != self.bytes_per_expert:
                raise ValueError(f"expert {e}: manifest accounts for {self.bytes_per_expert} "
                                 f"bytes but the region is {src.numel()}.")
            picked.append((e, src))
        if not picked:
            return 0
        if self.device.type != "cuda":
            for e, src in picked:
                self.stage_expert(e, src)
            return len(picked)
        if self._stage_buf is None:
            self._stage_buf = torch.empty((self.stage_rows, self.bytes_per_expert), dtype=torch.uint8,
                                          device=self.device)
        import ctypes
        from . import _lib
        base = len(self.stage)
        dsts = [self._stage_buf[base + i] for i in range(len(picked))]
        n = len(picked)
        dst = (ctypes.c_void_p * n)(*[d.data_ptr() for d in dsts])
        src = (ctypes.c_void_p * n)(*[t.data_ptr() for _, t in picked])
        size = (ctypes.c_size_t * n)(*[self.bytes_per_expert] * n)
        # the copy stream orders these writes after the previous token's admissions that
        # read the same buffers
        _lib.check(_lib.load().bigrig_copy_regions(
            dst, src, size, n, ctypes.c_void_p(self._copy_stream.cuda_stream)), "copy_regions")
        for (e, _), d in zip(picked, dsts):
            self.stage[e] = d
        self.stage_issued += n
        return n

    def stage_expert(self, e: int, blob) -> bool:
        """Copy expert e's bytes (pinned host) into a staging buffer ahead of its admission,
        on the copy stream; ``ensure`` admits a staged expert with a device-to-device copy.
        Returns False when there is nothing to do (resident, already staged, buffers full)."""
        e = int(e)
        if self.g2s[e] >= 0 or e in self.stage or len(self.stage) >= self.stage_rows:
            return False
        src = _as_u8(blob)
        if src.numel() != self.bytes_per_expert:
            raise ValueError(f"expert {e}: manifest accounts for {self.bytes_per_expert} bytes "
                             f"but the region is {src.numel()}.")
        if self._stage_buf is None:
            self._stage_buf = torch.empty((self.stage_rows, self.bytes_per_expert), dtype=torch.uint8,
                                          device=self.device)
        dst = self._stage_buf[len(self.stage)]
        if self.device.type == "cuda":
            # the copy stream orders this write after the previous token's admission that
            # read the same buffer
            with torch.cuda.stream(self._copy_stream):
                dst.copy_(src, non_blocking=src.is_pinned())
        else:
            dst.copy_(src)
        self.stage[e] = dst
        self.stage_issued += 1
        return True

    def admit_arrays(self, e: int, arrays, protect=(), _t0=None) -> int:
        """Write bytes already prepared (host or device) into a freed slot and record the
        admission (stream.py:757-780); returns the slot."""
        started = time.perf_counter() if _t0 is None else _t0
        slot = self._victim(protect=protect)
        self._write_slot(slot, arrays)
        self._placed(int(e), slot)
        self.admit_seconds += time.perf_counter() - started
        return slot

    def _write_slot(self, slot: int, src: torch.Tensor) -> None:
        n = self._bpe
        if self.device.type != "cuda":
            # host-side bookkeeping pools (tests): the stored bytes as they come
            self.slab[slot, :n].copy_(src.reshape(-1))
            return
        dst = self._landing_row(slot) if self._widen else self.slab[slot, :n]
        if self._batch is not None:
            self._batch.append((dst, src.reshape(-1), slot))
            return
        cs = self._copy_stream
        if self._reads_done is not None:
            cs.wait_event(self._reads_done)     # a kernel may still be reading this slot
        with torch.cuda.stream(cs):
            dst.copy_(src.reshape(-1), non_blocking=True)
            if src.device.type == "cuda":
                src.record_stream(cs)
        if self._widen:
            self._widen_slots([slot], cs)
        if self._copies_done is None:
            self._copies_done = torch.cuda.Event()
        self._copies_done.record(cs)
        self.admit_bytes += n

    def _landing_row(self, slot: int) -> torch.Tensor:
        """Device landing bytes of ``slot`` for experts stored in fewer bits than the slot
        holds (3-bit): they arrive here and are widened into the slot."""
        if self._landing is None:
            self._landing = torch.empty((self.capacity, self._bpe), dtype=torch.uint8,
                                        device=self.device)
        return self._landing[slot]

    def _widen_slots(self, slots, stream) -> None:
        lib = _lib.load()
        lp = ctypes.pointer(ops.c_layout(self.layout))
        st = ctypes.c_void_p(stream.cuda_stream)
        for slot in slots:
            _call(lib.bigrig_widen_expert(self._landing[slot].data_ptr(), self.slab[slot].data_ptr(),
                                          lp, self.layout.source_bits, st), "widen_expert")

    def _begin_writes(self) -> None:
        """Collect the slot writes of the admissions that follow (one decode step's)."""
        if self.device.type == "cuda":
            self._batch = []

    def _flush_writes(self) -> None:
        """Issue the collected slot writes on the copy stream: one wait on the slab's last
        reader, one library call with a cudaMemcpyAsync per slot, one completion event."""
        batch, self._batch = self._batch, None
        if not batch:
            return
        import ctypes
        from . import _lib
        cs = self._copy_stream
        if self._reads_done is not None:
            cs.wait_event(self._reads_done)     # a kernel may still be reading these slots
        n = len(batch)
        dst = (ctypes.c_void_p * n)(*[d.data_ptr() for d, _, _ in batch])
        src = (ctypes.c_void_p * n)(*[t.data_ptr() for _, t, _ in batch])
        size = (ctypes.c_size_t * n)(*[d.numel() for d, _, _ in batch])
        _lib.check(_lib.load().bigrig_copy_regions(dst, src, size, n,
                                                   ctypes.c_void_p(cs.cuda_stream)),
                   "copy_regions")
        if self._widen:
            self._widen_slots([slot for _, _, slot in batch], cs)
        stage = self._stage_buf
        for _, t, _ in batch:
            # device sources other than the pool's own staging buffers (which live as long
            # as the pool) must outlive the copy
            if t.device.type == "cuda" and (stage is None or t._base is not stage):
                t.record_stream(cs)
        if self._copies_done is None:
            self._copies_done = torch.cuda.Event()
        self._copies_done.record(cs)
        self.admit_bytes += sum(d.numel() for d, _, _ in batch)

    def ready(self, stream: torch.cuda.Stream | None = None) -> None:
        """Order ``stream`` (default: current) after every admission queued so far.

        Skipped while a CUDA graph is being captured: only a settled pool (see
        ``settle``) may be captured, and a capture cannot wait on outside events."""
        if self._copies_done is not None and self.device.type == "cuda":
            if torch.cuda.is_current_stream_capturing():
                return
            (stream or ops.current_stream(self._dev_index())).wait_event(self._copies_done)

    def mark_read(self, stream: torch.cuda.Stream | None = None) -> None:
        """Record that kernels reading the slab were queued on ``stream`` (default: current)."""
        if self.device.type == "cuda" and not torch.cuda.is_current_stream_capturing():
            if self._reads_done is None:
                self._reads_done = torch.cuda.Event()
            self._reads_done.record(stream or ops.current_stream(self._dev_index()))

    def _dev_index(self) -> int:
        """The slab's CUDA device as an int (a device object costs a lookup per call)."""
        i = getattr(self, "_dev_i", None)
        if i is None:
            i = self._dev_i = (self.device.index if self.device.index is not None
                               else torch.cuda.current_device())
        return i

    def settle(self) -> None:
        """Wait for every queued admission and kernel read; afterwards the pool's tables
        and slab are quiescent, which a CUDA-graph capture of a full pool requires."""
        if self.device.type == "cuda":
            if self._copy_stream is not None:
                self._copy_stream.synchronize()
            torch.cuda.current_stream(self.device).synchronize()
        self._copies_done = None
        self._reads_done = None

    def g2s_device(self) -> torch.Tensor:
        """The expert->slot table on the device, re-uploaded only when residency changed
        (from a small ring of pinned host buffers, each reused once its last upload ran)."""
        if self._g2s_dirty or self._g2s_dev is None:
            if self._g2s_dev is None or self.device.type != "cuda":
                t = torch.from_numpy(self.g2s.copy())
                if self._g2s_dev is None:
                    self._g2s_dev = t.to(self.device)
                else:
                    self._g2s_dev.copy_(t)
            else:
                ring = getattr(self, "_g2s_ring", None)
                if ring is None:
                    ring = self._g2s_ring = [
                        [torch.empty(self.n_experts, dtype=torch.int32).pin_memory(), None]
                        for _ in range(4)]
                    self._g2s_i = 0
                slot = ring[self._g2s_i]
                self._g2s_i = (self._g2s_i + 1) % len(ring)
                if slot[1] is not None:
                    slot[1].synchronize()
                else:
                    slot[1] = torch.cuda.Event()
                slot[0].numpy()[:] = self.g2s
                self._g2s_dev.copy_(slot[0], non_blocking=True)
                slot[1].record(ops.current_stream(self._dev_index()))
            self._g2s_dirty = False
        return self._g2s_dev

    def stats(self) -> dict:
        d = super().stats()
        d["resident_bytes"] = self.nbytes()
        return d


def _pair_chunks(sorted_experts: np.ndarray, C: int):
    """Spans of expert-sorted pairs holding at most C distinct experts (stream.py:1098-1126)."""
    uniq, starts = np.unique(sorted_experts, return_index=True)
    n = int(sorted_experts.shape[0])
    return [(int(starts[i]), int(starts[i + C]) if i + C < len(uniq) else n)
            for i in range(0, len(uniq), C)]


class StreamingSwitchGLU:
    """Drop-in for mlx_lm's SwitchGLU that computes over a pool's HBM slots (stream.py:814).

    ``__call__(x, indices) -> y[..., k, H]``: ``x`` bf16 ``[..., H]`` and ``indices``
    integer ``[..., k]`` on the pool's device.  Router weights are applied by the
    caller.  Raises ValueError when top-k exceeds the capacity (stream.py:1462-1465)
    and RuntimeError when one step needs more distinct misses than slots
    (stream.py:952-956).
    """

    def __init__(self, pool: ExpertPool, fetcher, activation=None, quantized: bool = True,
                 qparams: dict | None = None):
        if not quantized:
            raise NotImplementedError("only affine-quantised experts are built")
        # the activation is the model's (stream.py:827): SiLU / SwiGLU by default,
        # "gpt_oss" (gated) or "relu2" (plain fc1/fc2 experts); the kernels read it from
        # the layout, so the pool computes with it from here on
        if activation is not None and not isinstance(activation, str):
            activation = getattr(activation, "__name__", None) or type(activation).__name__
        name = {"SwiGLU": "swiglu", "silu": "silu", "swiglu": "swiglu"}.get(activation, activation)
        pool.layout = pool.layout.with_activation(name)
        self._pool = pool
        self._fetcher = fetcher
        self._q = dict(qparams or pool.spec_quant)
        self.fetch_seconds = 0.0
        self.fetch_bytes = 0
        self.chunked_calls = 0
        self.views_calls = 0
        self.sync_seconds = 0.0
        self.bypass = False
        self._sync_free = False
        self.same_answers = True
        self._held = None
        self._ahead = []
        self._then = None
        self.prefill_routed = None
        self._next = None
        self._next_gate = None
        self._pred_m = 0
        self._pred_budget = 0
        self.pred_issued = 0
        self.reroutes = 0
        self.reroute_lost = 0.0
        self.workspace = None

    # -- residency ----------------------------------------------------------
    def ensure(self, indices, ranks=None) -> np.ndarray:
        """Make every requested expert resident; return the slot-remapped indices
        (stream.py:922-978).  ``ranks`` overrides the rank read off the last axis."""
        gi = np.asarray(indices).astype(np.int64)
        k = gi.shape[-1] if gi.ndim else 1
        row = gi.reshape(-1).tolist()
        if ranks is None and len(row) == k and len(set(row)) == k:
            # one token (decode): its k distinct experts, ascending, each at its own rank
            order = sorted(range(k), key=row.__getitem__)
            uniq = np.array([row[j] for j in order], dtype=np.int64)
            best = np.array(order, dtype=np.int64)
        else:
            rk = (np.asarray(ranks, dtype=np.int64).reshape(-1) if ranks is not None
                  else np.tile(np.arange(k, dtype=np.int64), len(row) // max(1, k)))
            # each distinct expert once, ascending, at the best (lowest) rank it was asked at
            uniq, which = np.unique(np.asarray(row, dtype=np.int64), return_inverse=True)
            best = np.full(uniq.shape[0], np.iinfo(np.int64).max, dtype=np.int64)
            np.minimum.at(best, which.reshape(-1), rk)
        pool = self._pool
        need = pool.touch(uniq, best)
        protect = set(uniq.tolist())
        if need:
            if len(need) > pool.capacity:
                raise RuntimeError(
                    f"layer {pool.layer}: this step misses {len(need)} distinct experts and the "
                    f"pool has {pool.capacity} slots, so one would evict another before use; "
                    f"the capacity must be at least top-k (call with fewer tokens per step).")
            staged = [int(e) for e in need if int(e) in pool.stage]
            cold = [int(e) for e in need if int(e) not in pool.stage]
            pool._begin_writes()
            try:
                for e in staged:
                    pool.admit_arrays(e, pool.stage[e], protect=protect)
                    pool.stage_hits += 1
                if cold:
                    t0 = time.perf_counter()
                    blobs = self._fetch([(pool.layer, e) for e in cold])
                    self.fetch_seconds += time.perf_counter() - t0
                    for e in cold:
                        b = blobs[(pool.layer, e)]
                        self.fetch_bytes += pool.bytes_per_expert
                        pool.admit(e, b, protect=protect)
            finally:
                pool._flush_writes()
        pool.stage = {}
        return pool.g2s[gi]

    def _readback(self, x2: torch.Tensor, indices: torch.Tensor, k: int):
        """The routing on the host (the step's synchronisation point, stream.py:1447-1450),
        plus -- when staging is on -- the next layer's own router's top experts for this
        token, computed on the device and read back in the same synchronisation
        (stream.py:1428-1440)."""
        nxt = self._next
        if (STAGING and nxt is not None and self._next_gate is not None and x2.shape[0] == 1
                and not nxt.full):
            gw, gb = self._next_gate
            nk = min(STAGE_MAX, k, nxt.n_experts)
            pidx, _ = ops.router_topk(ops.router_logits(x2, gw, gb), nk)
            both = torch.cat([indices.reshape(1, k).to(torch.int32), pidx.reshape(1, nk)], dim=1)
            t0 = time.perf_counter()
            host = both.to("cpu").numpy().astype(np.int64)
            self.sync_seconds += time.perf_counter() - t0
            return host[:, :k], host[0, k:]
        t0 = time.perf_counter()
        gi = indices.reshape(-1, k).to("cpu").numpy().astype(np.int64)
        self.sync_seconds += time.perf_counter() - t0
        return gi, None

    def decode_layer(self, x: torch.Tensor, gate_w: torch.Tensor, gate_b: torch.Tensor | None,
                     k: int, mode: str, norm_topk: bool,
                     residual: torch.Tensor | None = None) -> torch.Tensor:
        """One decode token through the whole MoE block over this pool: the router's top-k
        is computed and read back (with, when staging is on, the next layer's prediction
        from the same two launches: one logits call over both routers' weights and one top-k
        over the two rows), made resident, then one library call computes the experts and
        the combine on that same routing (``bigrig_moe_layer_routed``: the persistent kernel
        without its router phase).  Returns out [1, H] = residual + sum_j score * y."""
        pool = self._pool
        H = x.shape[-1]
        if k > pool.capacity:
            raise ValueError(
                f"layer {pool.layer}: top-k is {k} but the pool holds {pool.capacity}. A single "
                f"token cannot be served, so no capacity below top-k is ever valid.")
        x2 = x.reshape(-1, H)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x2 = x2.contiguous()
        nxt = self._next
        E = pool.n_experts
        pred = None
        rs = self._route_scratch(x2.device, E, k)
        if not x2.is_cuda:
            ops._require_cuda("x", x2, torch.bfloat16)
        mcode = ops._MODES.get(mode)
        if mcode is None:
            raise ValueError(f"mode must be one of {tuple(ops._MODES)}, got {mode!r}")
        lib = _lib.load()
        dev = x2.get_device()
        st = ops._raw_stream(dev)
        self._check_weights(gate_w, gate_b)
        # the library called directly: every pointer here is a buffer of this layer's, checked
        # once, and x2 is bf16, contiguous and on the device (made so above)
        if (STAGING and nxt is not None and self._next_gate is not None and not nxt.full
                and nxt.n_experts == E and k <= E):
            w2, b2 = self._route_pair(gate_w, gate_b)
            _call(lib.bigrig_router_logits(x2.data_ptr(), w2.data_ptr(), b2.data_ptr(), rs[4], 1,
                                           H, 2 * E, st), "router_logits")
            _call(lib.bigrig_router_topk(rs[4], _lib.F32, 2, E, k, mcode, int(norm_topk), rs[5],
                                         rs[6], st), "router_topk")
            t0 = time.perf_counter()
            rs[3].copy_(rs[1])                                    # the host readback
            host = rs[3].numpy().astype(np.int64)
            self.sync_seconds += time.perf_counter() - t0
            gi, pred = host[:1], host[1]
        else:
            _call(lib.bigrig_router_logits(x2.data_ptr(), gate_w.data_ptr(),
                                           0 if gate_b is None else gate_b.data_ptr(), rs[4], 1,
                                           H, E, st), "router_logits")
            _call(lib.bigrig_router_topk(rs[4], _lib.F32, 1, E, k, mcode, int(norm_topk), rs[5],
                                         rs[6], st), "router_topk")
            t0 = time.perf_counter()
            rs[3][:1].copy_(rs[1][:1])                            # the host readback
            gi = rs[3][:1].numpy().astype(np.int64)
            self.sync_seconds += time.perf_counter() - t0
        self._count_routing(gi.reshape(-1))
        self.ensure(gi)
        pool.ready()
        if residual is not None and not (residual.is_cuda and residual.dtype == torch.bfloat16
                                         and residual.is_contiguous()
                                         and residual.numel() == H):
            ops._require_cuda("residual", residual, torch.bfloat16)
            raise ValueError(f"residual holds {residual.numel()} values, the layer makes {H}")
        ws = self.workspace or ops.default_workspace(x2.device)
        buf = ws.reserve(ops.workspace_bytes(1, k, E, pool.layout))
        out = torch.empty(1, H, dtype=torch.bfloat16, device=x2.device)
        # the routing read back above is the one computed: the layer runs on it (row 0 of the
        # device buffers) instead of routing a second time
        _call(lib.bigrig_moe_layer_routed(
            x2.data_ptr(), rs[5], rs[6], 1, E, k, pool.g2s_device().data_ptr(),
            pool.slab.data_ptr(), self._layout_ptr(), 0 if residual is None else residual.data_ptr(),
            out.data_ptr(), buf.data_ptr(), buf.numel(), st), "moe_layer_routed")
        pool.mark_read()
        if pred is not None:
            self._speculate(pred)
        return out

    def _route_scratch(self, device, E: int, k: int):
        """Per-layer routing buffers of the one-token path, made once: logits fp32 [2E] (this
        layer's and the next router's), indices int32 [2, k], scores fp32 [2, k] on the
        device, a pinned int32 [2, k] host copy for the readback, and the three device
        buffers' addresses."""
        rs = getattr(self, "_rs", None)
        if rs is None or rs[0].numel() != 2 * E or rs[1].shape[1] != k or rs[0].device != device:
            t = (torch.empty(2 * E, dtype=torch.float32, device=device),
                 torch.empty(2, k, dtype=torch.int32, device=device),
                 torch.empty(2, k, dtype=torch.float32, device=device),
                 torch.empty(2, k, dtype=torch.int32).pin_memory())
            rs = self._rs = t + (t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr())
        return rs

    def _check_weights(self, gate_w: torch.Tensor, gate_b: torch.Tensor | None) -> None:
        """The router's weights as the library wants them, checked once per pair of tensors."""
        key = (id(gate_w), gate_w.data_ptr(), None if gate_b is None else (id(gate_b), gate_b.data_ptr()))
        if getattr(self, "_checked", None) != key:
            ops._require_cuda("gate_w", gate_w, torch.bfloat16)
            if gate_b is not None:
                ops._require_cuda("gate_b", gate_b, torch.float32)
            ops._require_cuda("slab", self._pool.slab, torch.uint8)
            self._checked = key

    def _layout_ptr(self):
        """A ctypes pointer to this pool's layout struct (checked by the library once)."""
        lp = getattr(self, "_lp", None)
        if lp is None or lp[0] is not self._pool.layout:
            lp = self._lp = (self._pool.layout, ctypes.pointer(ops.c_layout(self._pool.layout)))
        return lp[1]

    def _route_pair(self, gate_w: torch.Tensor, gate_b: torch.Tensor | None):
        """This layer's and the next layer's router weights stacked [2E, H] (and biases),
        built once."""
        key = (gate_w.data_ptr(), None if gate_b is None else gate_b.data_ptr())
        if getattr(self, "_pair_key", None) != key:
            ngw, ngb = self._next_gate
            E = gate_w.shape[0]
            dev = gate_w.device
            zb = torch.zeros(E, dtype=torch.float32, device=dev)
            self._pair_w = torch.cat([gate_w, ngw]).contiguous()
            self._pair_b = torch.cat([gate_b if gate_b is not None else zb,
                                      ngb if ngb is not None else zb]).contiguous()
            self._pair_key = key
        return self._pair_w, self._pair_b

    def _speculate(self, predicted) -> None:
        """Stage the experts the next layer is likely to want while this layer computes
        (stream.py:1036-1072): those not resident in the next pool, at most STAGE_MAX, copied
        from pinned host DRAM behind this layer's own admissions.  Nothing here can change an
        answer: the next layer's ``ensure`` still admits exactly what its router selected, a
        staged one by a device-to-device copy and any other from the host."""
        nxt = self._next
        want = [int(e) for e in predicted if nxt.g2s[int(e)] < 0 and int(e) not in nxt.stage]
        want = want[:max(0, nxt.stage_rows - len(nxt.stage))]
        if not want:
            return
        blobs = self._fetch([(nxt.layer, e) for e in want])
        self.pred_issued += nxt.stage_experts([(e, blobs[(nxt.layer, e)]) for e in want])

    def _fetch(self, keys) -> dict:
        local = getattr(self._fetcher, "fetch_local", None)
        blobs = local(keys) if local is not None else None
        return self._fetcher.fetch(keys) if blobs is None else blobs

    def refresh(self) -> bool:
        """Re-decide whether this layer can skip the host round-trip (stream.py:1579-1603)."""
        self._sync_free = self._pool.full
        return self._sync_free

    # -- compute ------------------------------------------------------------
    def _run(self, x2: torch.Tensor, idx2: torch.Tensor, g2s: torch.Tensor | None,
             out: torch.Tensor | None = None) -> torch.Tensor:
        pool = self._pool
        pool.ready()
        y = ops.switch_glu(x2, idx2, pool.slab, pool.layout, pool.n_experts, g2s=g2s, out=out,
                           workspace=self.workspace)
        pool.mark_read()
        return y

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        pool = self._pool
        H = x.shape[-1]
        k = indices.shape[-1]
        lead = tuple(indices.shape[:-1])
        x2 = x.reshape(-1, H)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x2 = x2.contiguous()
        if self._sync_free or self.bypass:
            idx2 = indices.reshape(-1, k).to(torch.int32)
            if self.bypass:                      # timing control: slots scrambled, output wrong
                idx2 = torch.remainder(idx2, pool.capacity).contiguous()
                y = self._run(x2, idx2, None)
            else:
                y = self._run(x2, idx2.contiguous(), pool.g2s_device())
            return y.reshape(*lead, k, H)
        if k > pool.capacity:
            raise ValueError(
                f"layer {pool.layer}: top-k is {k} but the pool holds {pool.capacity}. A single "
                f"token cannot be served, so no capacity below top-k is ever valid.")
        gi, pred = self._readback(x2, indices, k)
        self._count_routing(gi.reshape(-1))
        if len(np.unique(gi)) <= pool.capacity:
            self.ensure(gi)
            idx2 = indices.reshape(-1, k).to(torch.int32).contiguous()
            y = self._run(x2, idx2, pool.g2s_device())
            if pred is not None:
                # after this layer's kernels are queued: the host work of staging overlaps
                # them instead of delaying their launch
                self._speculate(pred)
            return y.reshape(*lead, k, H)
        # More distinct experts than slots: expert-sorted spans of <= C experts, each made
        # resident and computed before the next span may evict it (stream.py:1509-1561).
        self.chunked_calls += 1
        pe = gi.reshape(-1)
        order = np.argsort(pe, kind="stable")
        spe = pe[order]
        tok = order // k
        rank = order % k
        y = torch.empty(pe.shape[0], H, dtype=torch.bfloat16, device=x2.device)
        spans = _pair_chunks(spe, pool.capacity)
        # Each span's experts renumbered 0..U-1 (sorted pairs: the rank among the span's
        # distinct experts) with a span-local expert->slot table, so that the expert GEMM
        # sees U experts sharing the span's rows -- its token tile follows the real rows per
        # expert -- instead of all E.  Host tables for every span go up in one copy.
        local = np.empty(spe.shape[0], dtype=np.int32)
        n_loc = []
        for lo, hi in spans:
            uniq, inv = np.unique(spe[lo:hi], return_inverse=True)
            local[lo:hi] = inv
            n_loc.append(len(uniq))
        order_dev = torch.from_numpy(order).to(x2.device)
        tok_dev = torch.from_numpy(tok).to(x2.device)
        local_dev = torch.from_numpy(local).to(x2.device)
        # The expert kernel is the one the whole call would take (the library's rule on its
        # pairs and all E experts: the GEMM beyond 32 pairs), forced for every span: both kernels are batch-invariant, so the
        # spans then give the whole call's bits (a span's own size could pick the other).
        mode, min_rows = _lib.get_path()
        forced = None
        if mode in ("auto", "chain"):
            P, E = pe.shape[0], pool.n_experts
            forced = "gemm" if P > 32 or P >= min_rows * min(P, E) else "gemv"
            _lib.set_path(forced, min_rows)
        try:
            for (lo, hi), u in zip(spans, n_loc):
                self.ensure(spe[lo:hi], ranks=rank[lo:hi])
                g2s_loc = torch.from_numpy(pool.g2s[np.unique(spe[lo:hi])].astype(np.int32)).to(x2.device)
                rows = x2.index_select(0, tok_dev[lo:hi]).contiguous()
                pool.ready()
                part = ops.switch_glu(rows, local_dev[lo:hi].reshape(-1, 1).contiguous(), pool.slab,
                                      pool.layout, u, g2s=g2s_loc, workspace=self.workspace)
                pool.mark_read()
                y.index_copy_(0, order_dev[lo:hi], part.reshape(hi - lo, H))
        finally:
            if forced is not None:
                _lib.set_path(mode, min_rows)
        return y.reshape(*lead, k, H)

    # -- prefill holding / read-ahead (stream.py:1174-1235) ----------------------
    def _count_routing(self, pe) -> None:
        if self._held is not None:
            np.add.at(self.prefill_routed, np.asarray(pe, dtype=np.int64), 1)

    @contextlib.contextmanager
    def holding(self, then=None):
        """The scope of one layer's pass over every prefill chunk.  Routed experts are
        tallied (``prefill_routed``, which ``StreamHandle.rewarm`` ranks), ``then`` --
        normally the next layer's read-ahead -- is kept for after the first chunk, and on
        exit whatever this layer queued for reading ahead is dropped."""
        self.prefill_routed = np.zeros(self._pool.n_experts, dtype=np.int64)
        self._held, self._then = {}, then
        try:
            yield self
        finally:
            self._held = self._then = None
            queued, self._ahead = self._ahead, []
            if queued:
                self._fetcher.drop(queued)

    def read_ahead(self) -> None:
        """Ask the fetcher to start reading all of this layer's experts.  A fetcher that
        refuses (closed, or too much already pending) is not an error: prefill still
        fetches on demand."""
        layer = self._pool.layer
        wanted = [(layer, e) for e in range(self._pool.n_experts)]
        try:
            self._fetcher.prefetch(wanted)
        except RuntimeError:
            return
        self._ahead = wanted


class StreamHandle:
    """Warm, measure and tear down a set of streamed layers (stream.py:1961-2200)."""

    def __init__(self, model, pools, mods, fetcher, manifest=None, full_layers=()):
        self.model, self.pools, self.mods = model, pools, mods
        self.fetcher, self.manifest = fetcher, manifest or {}
        self.full_layers = list(full_layers)

    def release_prefill(self) -> None:
        """Drop every layer's outstanding read-ahead."""
        for m in self.mods:
            queued, m._ahead = m._ahead, []
            if queued and m._fetcher is not None:
                m._fetcher.drop(queued)

    def rewarm(self, per_layer: int) -> int:
        """Ask the fetcher to refresh, per streamed layer, the ``per_layer`` experts the
        last prefill routed most (ties to the lower id; never-routed experts are skipped).
        Returns what the fetcher reports."""
        keys = []
        layers = {m._pool.layer: m.prefill_routed for m in self.mods
                  if m._pool is not None and m.prefill_routed is not None}
        for layer in sorted(layers):
            counts = layers[layer]
            ranked = np.lexsort((np.arange(counts.shape[0]), -counts))[:per_layer]
            keys.extend((layer, int(e)) for e in ranked if counts[e] > 0)
        return self.fetcher.refresh(keys) if keys else 0

    def prefill_layer(self, layer: int, read_ahead: bool = False):
        """Context held while layer-major prefill runs every chunk through ``layer``
        (stream.py:2009-2034).  Whole layers (capacity == experts) get a no-op scope."""
        by_layer = {m._pool.layer: m for m in self.mods
                    if m._pool is not None and m._pool.capacity < m._pool.n_experts}
        m = by_layer.get(layer)
        nxt = by_layer.get(layer + 1) if read_ahead else None
        if m is None:
            if nxt is not None:
                nxt.read_ahead()
            return contextlib.nullcontext()
        return m.holding(then=nxt.read_ahead if nxt is not None else None)

    def warm(self, mode="auto"):
        """Fill the pools: "auto" fills only pools with C == E, "full" all, "lazy" none
        (stream.py:2036-2073)."""
        if mode not in ("auto", "full", "lazy", True, False):
            raise ValueError(f"warm mode must be auto/full/lazy, got {mode!r}")
        mode = {True: "full", False: "lazy"}.get(mode, mode)
        if mode == "lazy":
            return self
        for p in self.pools:
            if mode == "auto" and p.capacity < p.n_experts:
                p.hits = p.misses = 0
                continue
            blobs = self.fetcher.fetch([(p.layer, e) for e in range(p.capacity)])
            for e in range(p.capacity):
                p.touch([e], [0])
                p.admit(e, blobs[(p.layer, e)])
            p.hits = p.misses = 0
        return self

    def usage(self) -> dict:
        """Requests per expert in this run, keyed ``"layer:expert"`` (the usage-file format)."""
        return {f"{m._pool.layer}:{e}": int(m._pool.uses[e])
                for m in self.mods for e in np.flatnonzero(m._pool.uses)}

    def save_usage(self, path: str, decay: float = 0.5) -> str:
        """Write the usage file at ``path``: earlier counts there scaled by ``decay`` and
        truncated (entries reaching 0 are dropped), plus this run's counts.  The file is
        replaced atomically (stream.py:2084-2105)."""
        try:
            with open(path) as fh:
                earlier = json.load(fh) or {}
        except (OSError, ValueError):
            earlier = {}
        totals = {}
        for key, n in earlier.items():
            kept = int(n * decay)
            if kept > 0:
                totals[key] = kept
        for key, n in self.usage().items():
            totals[key] = totals.get(key, 0) + n
        folder = os.path.dirname(path)
        if folder:
            os.makedirs(folder, exist_ok=True)
        part = f"{path}.tmp"
        with open(part, "w") as fh:
            json.dump(totals, fh)
        os.replace(part, path)
        return path

    def resident_gb(self) -> float:
        return sum(p.nbytes() for p in self.pools) / 1e9

    def stats(self) -> dict:
        """Counters summed over the streamed layers."""
        pools, mods = self.pools, self.mods
        hits = sum(p.hits for p in pools)
        misses = sum(p.misses for p in pools)
        capped = [p.capacity for p in pools if p.capacity < p.n_experts]
        out = dict(layers=len(pools),
                   full_layers=sum(p.capacity == p.n_experts for p in pools),
                   sync_free=sum(bool(m._sync_free) for m in mods),
                   hits=hits, misses=misses,
                   miss_rate=misses / (hits + misses) if hits + misses else 0.0,
                   capacity=min(capped) if capped else (pools[0].capacity if pools else 0),
                   n_experts=pools[0].n_experts if pools else 0,
                   resident_gb=self.resident_gb(),
                   admit_gb=sum(p.admit_bytes for p in pools) / 1e9)
        for key, attr in (("fetch_seconds", "fetch_seconds"), ("sync_seconds", "sync_seconds"),
                          ("chunked_calls", "chunked_calls")):
            out[key] = sum(getattr(m, attr) for m in mods)
        out["admit_seconds"] = sum(m._pool.admit_seconds for m in mods)
        out["stage_issued"] = sum(p.stage_issued for p in pools)
        out["stage_hits"] = sum(p.stage_hits for p in pools)
        return out

    def reset_stats(self):
        for p in self.pools:
            p.hits = p.misses = 0
            p.stage_issued = p.stage_hits = 0
            p.admit_seconds = 0.0
            p.admit_bytes = 0
        for m in self.mods:
            m.fetch_seconds = 0.0
            m.sync_seconds = 0.0
            m.fetch_bytes = 0
        return self

    def close(self) -> None:
        """Release every slab explicitly (stream.py:2160-2191)."""
        for p in self.pools:
            p.slab = None
            p._stage_buf = None
            p.stage = {}
            p._built = False
        for m in self.mods:
            m._pool = None
            m._fetcher = None
        self.pools, self.mods = [], []
        try:
            self.fetcher.close()
        except Exception:  # noqa: BLE001 -- teardown must not raise
            pass


def attach(blocks, store, capacity, policy: str = "lfuda", full_layers=(), warm=True,
           device=None) -> StreamHandle:
    """Give each MoE block a pool-backed StreamingSwitchGLU over ``store`` (stream.py:1842-1958).

    ``blocks``: list of objects with ``layer``, ``n_experts``, ``spec``, ``quant`` and a
    ``switch`` attribute to replace.  ``capacity`` is an int or a fraction of E in (0, 1].
    """
    full = set(full_layers or ())
    pools, mods = [], []
    dev = torch.device(device) if device is not None else (
        torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else None)
    # one copy stream for every layer: a layer's staging of the next layer's experts queues
    # behind its own admissions, and the next layer's admission from staging behind both
    copy_stream = torch.cuda.Stream(device=dev) if dev is not None and dev.type == "cuda" else None
    for blk in blocks:
        E = blk.n_experts
        if blk.layer in full:
            C = E
        else:
            C = int(round(capacity * E)) if isinstance(capacity, float) and capacity <= 1.0 \
                else int(capacity)
        C = max(1, min(E, C))
        pool = ExpertPool(blk.layer, None, E, C, blk.spec, policy=policy, quant=blk.quant,
                          device=device, copy_stream=copy_stream).build()
        mod = StreamingSwitchGLU(pool, store)
        blk.switch = mod
        pools.append(pool)
        mods.append(mod)
    # every streamed layer knows the next one's router (stream.py:1895-1911)
    for j, mod in enumerate(mods[:-1]):
        gw = getattr(blocks[j + 1], "gate_w", None)
        if gw is not None:
            mod._next = pools[j + 1]
            mod._next_gate = (gw, getattr(blocks[j + 1], "gate_b", None))
            mod._pred_m = STAGE_MAX
    h = StreamHandle(blocks, pools, mods, store, full_layers=sorted(full))
    h.warm(warm if warm is not True else "auto")
    for m in mods:
        m.refresh()
    return h


__all__ = ["ExpertPool", "StreamingSwitchGLU", "StreamHandle", "attach", "PROJECTIONS",
           "MLP_PROJECTIONS",
           "projections_of", "is_gated"]
