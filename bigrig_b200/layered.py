"""Layer-major prefill: every prompt chunk through layer L before any chunk reaches L+1.

Restates the schedule of bigrig_engine/layered.py:85-131.  Chunk boundaries are
``step`` tokens counted from the first token, as the chunked loop counts them;
only the order of independent work changes, so each chunk's result is the one
chunk-major order gives.  ``layer_scope(i)``, if given, returns a context held
while layer i runs every chunk -- StreamHandle.prefill_layer uses it to count
the layer's routing and start the next layer's read-ahead.  With streamed
experts this visits each layer's experts once per prompt instead of once per
chunk, and on the B200 it puts every chunk's rows for an expert behind one
resident copy.

The reference checks a model-specific forward hash (Qwen3.5) before using the
schedule; here the layers are plain callables ``h -> h'`` and the caller vouches
that each depends only on its own chunk (true of the MoE stack; a model with
attention passes layers that own their KV cache).
"""
from __future__ import annotations

import contextlib


def chunks(x, step: int) -> list:
    """x[T, ...] cut into [step, ...] pieces from the first token."""
    if step < 1:
        raise ValueError(f"step must be >= 1, got {step}")
    return [x[i:i + step] for i in range(0, x.shape[0], step)]


def prefill(layers, hidden: list, layer_scope=None, progress=None, token_wise: bool = False) -> list:
    """Run every chunk of ``hidden`` through ``layers`` layer by layer; returns the chunks.

    ``token_wise``: the caller vouches that every layer treats each token on its own (an
    MoE stack without attention), so a layer runs once over all chunks' tokens stacked
    and the result is cut back into the same chunks.  The rows and every token's result
    are those of the chunked loop; the expert GEMMs get all the prompt's rows of an
    expert at once instead of one chunk's share."""
    hidden = list(hidden)
    n = len(layers)
    if not hidden or n == 0:
        return hidden
    sizes = [h.shape[0] for h in hidden]
    total = sum(sizes)
    if token_wise and len(hidden) > 1:
        import torch
        stacked = torch.cat(hidden)
        for li, layer in enumerate(layers):
            with layer_scope(li) if layer_scope is not None else contextlib.nullcontext():
                stacked = layer(stacked)
            if progress is not None:
                progress(total * (li + 1) // n, total)
        return list(torch.split(stacked, sizes))
    for li, layer in enumerate(layers):
        with layer_scope(li) if layer_scope is not None else contextlib.nullcontext():
            for j in range(len(hidden)):
                hidden[j] = layer(hidden[j])
        if progress is not None:
            progress(total * (li + 1) // n, total)
    return hidden
