"""Layer-major prefill (bigrig_engine/layered.py:85-131): chunks cut from the first token,
every chunk through layer L before layer L+1, and the token-wise schedule that runs a
layer once over all chunks.  Host logic on CPU tensors."""
import torch

from bigrig_b200 import layered


def _layers(log):
    def mk(i, fn):
        def layer(h):
            log.append((i, h.shape[0]))
            return fn(h)
        return layer
    return [mk(0, lambda h: h * 2 + 1), mk(1, torch.tanh), mk(2, lambda h: h.cumsum(dim=1))]


def test_chunks_count_from_first_token():
    x = torch.arange(17).view(17, 1)
    got = layered.chunks(x, 5)
    assert [c.shape[0] for c in got] == [5, 5, 5, 2]
    assert torch.equal(torch.cat(got), x)


def test_layer_major_order_and_results():
    x = torch.randn(17, 4)
    log = []
    out = layered.prefill(_layers(log), layered.chunks(x, 5))
    assert log == [(li, n) for li in range(3) for n in (5, 5, 5, 2)]
    want = torch.tanh(x * 2 + 1).cumsum(dim=1)
    assert torch.equal(torch.cat(out), want)


def test_token_wise_runs_each_layer_once_with_the_same_result():
    x = torch.randn(17, 4)
    log, scopes, prog = [], [], []

    class Scope:
        def __init__(self, i):
            self.i = i

        def __enter__(self):
            scopes.append(self.i)

        def __exit__(self, *a):
            return False

    chunked = layered.prefill(_layers([]), layered.chunks(x, 5))
    tw = layered.prefill(_layers(log), layered.chunks(x, 5), layer_scope=Scope,
                         progress=lambda d, t: prog.append((d, t)), token_wise=True)
    assert log == [(0, 17), (1, 17), (2, 17)]
    assert scopes == [0, 1, 2]
    assert prog == [(5, 17), (11, 17), (17, 17)]
    assert [c.shape[0] for c in tw] == [5, 5, 5, 2]
    for a, b in zip(chunked, tw):
        assert torch.equal(a, b)


def test_empty_inputs():
    assert layered.prefill(_layers([]), []) == []
    x = torch.randn(3, 2)
    out = layered.prefill([], [x], token_wise=True)
    assert len(out) == 1 and out[0] is x
