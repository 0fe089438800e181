"""Host side of the expert fetch: every expert's packed bytes in pinned host DRAM.

Replaces bigrig_engine/fetch.py's ParallelFetcher/WeightStore (fetch.py:161-779).
On Apple Silicon the reference reads expert regions from SSD into page-cache
memory the GPU can address directly.  A B200 cannot address host pages at HBM
speed, so the B200 design holds the model's experts in page-locked host memory
(one region per expert, in the packed order of formats.pack_expert) and admits a
missed expert with one asynchronous host->device copy on a side stream
(stream.ExpertPool).  The fetch interface keeps the reference's names and
meaning -- ``fetch(keys) -> {key: bytes}``, ``fetch_local``, ``prefetch``,
``warm``, ``drop``, ``refresh``, ``stats``, ``close`` -- where a key is
``(layer, expert)`` and the bytes are a pinned uint8 tensor view (no copy).
Everything is already in DRAM, so prefetch/warm/drop have nothing to move.
"""
from __future__ import annotations

import threading

import numpy as np
import torch

from .formats import bytes_per_expert, manifest_regions


class HostExpertStore:
    """Pinned host copy of every expert of every layer: ``[E, bytes_per_expert]`` per layer."""

    def __init__(self, layers: dict, pin: bool = True):
        """``layers``: {layer: (n_experts, bytes_per_expert)}."""
        self._lock = threading.Lock()
        self._closed = False
        self.layers = {}
        self.pinned = bool(pin) and torch.cuda.is_available()
        for li, (E, bpe) in layers.items():
            t = torch.empty((E, bpe), dtype=torch.uint8, pin_memory=self.pinned)
            self.layers[int(li)] = t
        self.hits = 0
        self.bytes_served = 0

    # -- construction -------------------------------------------------------
    @classmethod
    def from_blob(cls, blob_path: str, manifest: dict, pin: bool = True) -> "HostExpertStore":
        """Load a packed blob (``pack_experts`` format, stream.py:106-186) into pinned DRAM."""
        regions = manifest_regions(manifest)
        layers = {int(li): (int(info["n_experts"]), int(info["bytes_per_expert"]))
                  for li, info in manifest["layers"].items()}
        store = cls(layers, pin=pin)
        with open(blob_path, "rb") as f:
            for (li, e), (off, n) in sorted(regions.items(), key=lambda kv: kv[1][0]):
                want = layers[li][1]
                if n != want:
                    raise ValueError(f"region {li}:{e} is {n} bytes, the layer's experts are {want}")
                f.seek(off)
                buf = f.readinto(store.layers[li][e].numpy())
                if buf != n:
                    raise IOError(f"short read of {li}:{e}: {buf} of {n} bytes")
        return store

    @classmethod
    def from_direct(cls, model_dir_or_manifest, pin: bool = True) -> "HostExpertStore":
        """Load a model's experts straight from its safetensors shards (bigrig_engine/direct.py
        ``store``): ``model_dir_or_manifest`` is the model folder or ``direct.expert_manifest``'s
        result.  Each stacked component tensor is read once and scattered into place."""
        from . import direct
        man = (model_dir_or_manifest if isinstance(model_dir_or_manifest, dict)
               else direct.expert_manifest(model_dir_or_manifest))
        layers = {int(li): (int(info["n_experts"]), int(info["bytes_per_expert"]))
                  for li, info in man["layers"].items()}
        store = cls(layers, pin=pin)
        direct.fill_store(store, man)
        return store

    def put(self, layer: int, e: int, blob) -> None:
        """Write one expert's packed bytes (length-checked) into the store."""
        dst = self.layers[int(layer)][int(e)]
        src = blob if isinstance(blob, torch.Tensor) else torch.from_numpy(
            np.frombuffer(blob, dtype=np.uint8) if not isinstance(blob, np.ndarray) else blob)
        if src.numel() != dst.numel():
            raise ValueError(f"expert {layer}:{e}: {src.numel()} bytes, slots hold {dst.numel()}")
        dst.copy_(src.reshape(-1))

    # -- the reference's fetch interface --------------------------------------
    def _check(self):
        if self._closed:
            raise RuntimeError("fetcher is closed")

    def fetch(self, keys) -> dict:
        """{(layer, e): pinned uint8 tensor} for every key, no copy."""
        self._check()
        out = {}
        for li, e in keys:
            t = self.layers[int(li)][int(e)]
            out[(li, e)] = t
            self.bytes_served += t.numel()
        self.hits += len(out)
        return out

    def fetch_local(self, keys):
        return self.fetch(keys)

    def prefetch(self, keys) -> None:
        self._check()

    def warm(self, keys) -> None:
        self._check()

    def drop(self, keys) -> None:
        pass

    def refresh(self, keys) -> int:
        return 0

    def stats(self) -> dict:
        return {"served": self.hits, "bytes": self.bytes_served, "pinned": self.pinned,
                "host_bytes": sum(t.numel() for t in self.layers.values())}

    def close(self) -> None:
        self._closed = True
        self.layers = {}

    def layer_tensor(self, layer: int) -> torch.Tensor:
        return self.layers[int(layer)]


def store_for_spec(n_layers: int, n_experts: int, spec: dict, pin: bool = True) -> HostExpertStore:
    return HostExpertStore({li: (n_experts, bytes_per_expert(spec)) for li in range(n_layers)},
                           pin=pin)
