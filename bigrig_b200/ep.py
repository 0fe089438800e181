"""Expert parallelism across the GPUs of one node: all-to-all token dispatch and combine.

The reference runs on one Mac and has no distributed code; this is the B200
design's way of sharding its hot path.  Experts split into contiguous blocks, rank r
owning ``[r * E/G, (r + 1) * E/G)`` of every layer; tokens stay data-parallel (each
rank routes its own tokens with the replicated router).  One MoE layer is then

1. plan: each (token, k) pair goes to the rank owning its expert; pairs are grouped
   by destination with a stable sort, so a rank's rows arrive in the sender's
   (token, k) order;
2. dispatch: one ``all_to_all_single`` of the pair rows, each carrying its local
   expert id in the row's padding (``padded`` mode; the exact mode sends rows and ids
   separately);
3. the owner computes its experts over the received rows (k = 1 per row);
4. combine: the reverse ``all_to_all_single`` returns each pair's output to its
   sender, which applies the router weights (``sum_k score * y``).

Two exchange modes.  ``padded`` (decode): every peer block has a fixed capacity of
T*k rows (the most one rank can send to one peer), padding rows carry expert id -1
and are skipped by the kernels; no sizes cross to the host and every step is the same
sequence of device work, so a whole decode step can be captured in a CUDA graph
(``bench.py`` does).  ``exact`` (prefill): counts are exchanged first (int64 [G]),
then rows and ids with those split sizes.

Transport is NCCL over NVLink 5 / NVSwitch.  Nothing here issues TMA or multicast
loads; peer memory is only touched by NCCL.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class ExpertParallel:
    """Dispatch/combine of one MoE layer's pairs across the ranks of ``group``."""

    def __init__(self, n_experts: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if n_experts % self.world:
            raise ValueError(f"{n_experts} experts do not split evenly over {self.world} ranks")
        self.n_experts = n_experts
        self.per_rank = n_experts // self.world

    def local_range(self) -> tuple:
        return self.rank * self.per_rank, (self.rank + 1) * self.per_rank

    def plan(self, indices: torch.Tensor) -> dict:
        """Destination of every pair, pairs grouped by destination (stable), counts."""
        T, k = indices.shape
        flat = indices.reshape(-1).long()
        dest = torch.div(flat, self.per_rank, rounding_mode="floor")
        order = torch.sort(dest, stable=True).indices
        # a scatter-add, not bincount: bincount reads its input's maximum back to the host
        counts = torch.zeros(self.world, dtype=torch.int64, device=flat.device)
        counts.scatter_add_(0, dest, torch.ones_like(dest))
        return {"T": T, "k": k, "order": order, "tok": torch.div(order, k, rounding_mode="floor"),
                "local": (flat[order] - dest[order] * self.per_rank).to(torch.int32),
                "dest": dest[order], "counts": counts}

    # -------------------------------------------------------------- exchanges
    def _a2a(self, out, inp, out_splits=None, in_splits=None):
        if self.world == 1:
            out.copy_(inp)
            return out
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)
        return out

    def dispatch_combine(self, x: torch.Tensor, indices: torch.Tensor, scores: torch.Tensor,
                         expert_fn, padded: bool = True, combine_fn=None) -> torch.Tensor:
        """Combined output [T, H] of a layer whose experts are split over the group.

        ``expert_fn(rows [R, H], local_ids [R] int32) -> [R, H]`` computes this rank's
        experts (ids < 0 are padding: any output, never read).  ``combine_fn(y [T, k, H],
        scores) -> [T, H]`` applies the router weights (default: fp32 weighted sum in k
        order, stored in x's dtype)."""
        p = self.plan(indices)
        T, k = p["T"], p["k"]
        H = x.shape[1]
        G = self.world
        P = T * k
        rows = x.index_select(0, p["tok"])
        if padded:
            cap = P
            # position of each sorted pair inside its destination's block
            start = torch.cumsum(p["counts"], 0) - p["counts"]
            within = torch.arange(P, device=x.device) - start[p["dest"]]
            slot = p["dest"] * cap + within
            # one payload row per pair: its H values, then 16 bytes of padding whose first
            # word is the pair's local expert id (rows stay 16-byte aligned); padding rows
            # carry id -1
            es = x.element_size()
            if (H * es) % 4:
                raise ValueError(f"padded dispatch needs rows of whole 32-bit words, got "
                                 f"{x.dtype} [{H}]")
            W = H + 16 // es                           # 16 bytes of padding per row
            at = H * es // 4                           # the id's word
            words = torch.zeros(G * cap, W * es // 4, dtype=torch.int32, device=x.device)
            words[:, at] = -1
            words[:, at].index_copy_(0, slot, p["local"])
            send = words.view(x.dtype)                 # [G * cap, W]
            send[slot, :H] = rows
            recv = torch.empty_like(send)
            self._a2a(recv, send)
            recv_id = recv.view(torch.int32)[:, at].contiguous()
            y_recv = expert_fn(recv[:, :H].contiguous(), recv_id)
            back = torch.empty_like(y_recv)
            self._a2a(back, y_recv)
            y_sorted = back.index_select(0, slot)
        else:
            counts = p["counts"].to(torch.int64)
            recv_counts = torch.empty_like(counts)
            self._a2a(recv_counts, counts)
            in_splits = counts.tolist()
            out_splits = recv_counts.tolist()
            recv_x = torch.empty(sum(out_splits), H, dtype=x.dtype, device=x.device)
            recv_id = torch.empty(sum(out_splits), dtype=torch.int32, device=x.device)
            self._a2a(recv_x, rows, out_splits, in_splits)
            self._a2a(recv_id, p["local"], out_splits, in_splits)
            y_recv = expert_fn(recv_x, recv_id)
            y_sorted = torch.empty(P, H, dtype=y_recv.dtype, device=x.device)
            self._a2a(y_sorted, y_recv, in_splits, out_splits)
        y = torch.empty(P, H, dtype=y_sorted.dtype, device=x.device)
        y.index_copy_(0, p["order"], y_sorted)
        y = y.reshape(T, k, H)
        if combine_fn is not None:
            return combine_fn(y, scores)
        acc = torch.zeros(T, H, dtype=torch.float32, device=x.device)
        for j in range(k):
            acc = acc + scores[:, j:j + 1].float() * y[:, j].float()
        return acc.to(x.dtype)


def local_expert_fn(slab, layout, n_local: int, g2s=None, workspace=None):
    """``expert_fn`` over this rank's experts on the sm_100a kernels (one pair per row)."""
    from . import ops

    def fn(rows: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        y = ops.switch_glu(rows.contiguous(), ids.reshape(-1, 1).contiguous(), slab, layout,
                           n_local, g2s=g2s, workspace=workspace)
        return y.reshape(rows.shape[0], rows.shape[1])

    return fn


class PeerBuffers:
    """Every rank's expert-parallel peer buffer, mapped into this process
    (``bigrig_peer_group``): each rank allocates one buffer sized for ``tokens`` rows per
    layer call, the IPC handles are exchanged over the process group, and every other
    rank's buffer is opened here.  ``bigrig_peer_layer`` (``ops.peer_layer``) then moves
    rows between them with stores over NVLink; no NCCL call is on that path.  A group of
    one rank (no process group) is its own peer.  ``wait_ms`` bounds each wait for another
    rank (0: the library's 10 s).  ``lib`` replaces the loaded library (host-logic tests)."""

    def __init__(self, tokens: int, hidden: int, top_k: int, device, group=None,
                 wait_ms: int = 0, lib=None):
        import contextlib
        import ctypes

        from . import _lib
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device(device)
        lib = self._lib = lib if lib is not None else _lib.load()
        nbytes = lib.bigrig_peer_buffer_bytes(self.world, tokens, hidden, top_k)
        if nbytes == 0:
            raise ValueError(f"no peer group of {self.world} ranks x {tokens} tokens "
                             f"(at most {_lib.PEER_MAX_RANKS} ranks)")
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * _lib.PEER_HANDLE_BYTES)()
        on_device = (torch.cuda.device(self.device) if self.device.type == "cuda"
                     else contextlib.nullcontext())
        with on_device:
            _lib.check(lib.bigrig_peer_alloc(nbytes, ctypes.byref(own), handle), "peer_alloc")
            handles = [bytes(handle)]
            if self.world > 1:
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(handle), group=group)
            self._opened = []
            bases = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(own.value)
                    continue
                p = ctypes.c_void_p()
                buf = (ctypes.c_uint8 * _lib.PEER_HANDLE_BYTES).from_buffer_copy(h)
                _lib.check(lib.bigrig_peer_open(buf, ctypes.byref(p)), "peer_open")
                self._opened.append(p.value)
                bases.append(p.value)
        self._own = own.value
        self.c = _lib.PeerGroup(world=self.world, rank=self.rank, tokens=tokens, hidden=hidden,
                                top_k=top_k, wait_ms=int(wait_ms))
        for i, b in enumerate(bases):
            self.c.base[i] = b
        self.tokens, self.hidden, self.top_k = tokens, hidden, top_k
        if self.world > 1:
            dist.barrier(group)                  # every buffer mapped before the first layer

    def errors(self) -> int:
        """Read and clear this rank's count of peer waits that ran out."""
        import ctypes

        from . import _lib
        n = ctypes.c_int32(0)
        s = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(self._lib.bigrig_peer_errors(ctypes.byref(self.c), ctypes.byref(n),
                                                ctypes.c_void_p(s)), "peer_errors")
        return int(n.value)

    def close(self) -> None:
        """Unmap the other ranks' buffers and free this one (after every rank is done)."""
        if self._own is None:
            return
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(self.group)
        for p in self._opened:
            self._lib.bigrig_peer_close(p)
        if self.world > 1:
            dist.barrier(self.group)             # no rank frees while another still maps it
        self._lib.bigrig_peer_free(self._own)
        self._own = None
        self._opened = []
