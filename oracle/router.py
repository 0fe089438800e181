"""Router top-k / softmax and the token->expert permutation, restated in numpy.

TEST INFRASTRUCTURE ONLY.

Router (the mlx_lm MoE blocks are not in the reference tree; the routing rule is
summarised by bigrig_engine/adapter.py:74-92 and the predictor at
bigrig_engine/stream.py:1436-1439):

* ``softmax_topk``: probabilities = softmax over all E logits (fp32), the k
  largest are kept; optionally renormalised to sum to one (Qwen3-style
  ``norm_topk_prob``; OLMoE keeps them raw).
* ``topk_softmax``: the k largest logits are kept and the softmax runs over those
  k only (Mixtral, gpt-oss).

Selection is made on the logits, largest first, ties to the lower expert id, so
the returned order is the router rank (0 = highest scoring) that the pool's
policies read (bigrig_engine/pool.py:38-40).  MLX's ``argpartition`` returns an
implementation-defined order, so reference parity is on the sorted index set;
against this restatement the CUDA kernel is compared bit for bit.

Permutation (bigrig_engine/stream.py:1246-1250, 1275-1276): ``order`` is the
stable argsort of the flattened (token, k) expert ids, ``tok = order // k``,
``rank = order % k`` and the inverse is ``argsort(order)``.
"""
from __future__ import annotations

import numpy as np

MODES = ("softmax_topk", "topk_softmax")


def router_logits(x: np.ndarray, w: np.ndarray, bias=None) -> np.ndarray:
    """fp32 logits = x . W^T (+ bias), x [T, H] and W [E, H] given as fp32 values."""
    lg = (x.astype(np.float32) @ w.astype(np.float32).T).astype(np.float32)
    if bias is not None:
        lg = (lg + np.asarray(bias, dtype=np.float32)).astype(np.float32)
    return lg


def softmax(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.float32)
    m = v.max(axis=-1, keepdims=True)
    e = np.exp(v - m).astype(np.float32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def topk(logits: np.ndarray, k: int, mode: str = "softmax_topk", norm_topk: bool = False):
    """(indices int32 [T, k] in rank order, scores fp32 [T, k])."""
    if mode not in MODES:
        raise ValueError(f"mode must be one of {MODES}, got {mode!r}")
    lg = np.asarray(logits, dtype=np.float32)
    T, E = lg.shape
    if not 1 <= k <= E:
        raise ValueError(f"top_k must be in [1, {E}], got {k}")
    idx = np.argsort(-lg, axis=-1, kind="stable")[:, :k].astype(np.int32)
    if mode == "softmax_topk":
        p = softmax(lg)
        sc = np.take_along_axis(p, idx, axis=-1)
        if norm_topk:
            sc = (sc / sc.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    else:
        sc = softmax(np.take_along_axis(lg, idx, axis=-1))
    return idx, sc.astype(np.float32)


def permutation(indices: np.ndarray, n_experts: int) -> dict:
    """The stable expert-sorted permutation of (token, k) pairs and its bookkeeping."""
    ind = np.asarray(indices)
    k = ind.shape[-1]
    flat = ind.reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable")
    inv = np.argsort(order, kind="stable")
    counts = np.bincount(flat, minlength=n_experts)
    offsets = np.concatenate([[0], np.cumsum(counts)])
    seg_expert = np.nonzero(counts)[0]
    seg_start = offsets[seg_expert]
    return {"order": order.astype(np.int32), "inv": inv.astype(np.int32),
            "tok": (order // k).astype(np.int32), "rank": (order % k).astype(np.int32),
            "sorted_experts": flat[order].astype(np.int32),
            "offsets": offsets.astype(np.int32), "seg_expert": seg_expert.astype(np.int32),
            "seg_start": np.append(seg_start, len(flat)).astype(np.int32)}
