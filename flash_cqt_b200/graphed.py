"""CUDA-graph capture / replay of a per-slice function.

Drop-in for ``flash_cqt/graphed.py:35-57`` (``Graphed(fn, *example)``): warm
up on a side stream (so that lazy allocations and table uploads happen outside
the capture), capture one call on static input buffers, then every call copies
the new inputs in, replays the graph and clones the outputs out.  Inference
only -- capture does not record autograd.  The B200 entry points allocate
nothing and never synchronise, so the whole round trip is one graph launch.
"""
import torch


def _tensors(t):
    if torch.is_tensor(t):
        yield t
    elif isinstance(t, (list, tuple)):
        for u in t:
            yield from _tensors(u)


def _clone(t):
    if torch.is_tensor(t):
        return t.clone()
    if isinstance(t, (list, tuple)):
        return type(t)(_clone(u) for u in t)
    return t


class Graphed:
    def __init__(self, fn, *example, warmup=3):
        if not torch.cuda.is_available():
            raise RuntimeError("cuda graphs need a cuda device")
        self._fn = fn
        self._in = _clone(example)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(warmup):
                fn(*self._in)
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self._out = fn(*self._in)

    @property
    def static_inputs(self):
        """the captured input buffers (write into them, then call run())"""
        return list(_tensors(self._in))

    @property
    def static_outputs(self):
        return self._out

    def run(self):
        """replay on whatever the static inputs hold; returns static outputs"""
        self.graph.replay()
        return self._out

    @torch.no_grad()
    def replay(self, *args):
        """copy the inputs in and replay; returns the static outputs (not
        cloned -- the next replay overwrites them)"""
        for dst, src in zip(_tensors(self._in), _tensors(args)):
            dst.copy_(src)
        self.graph.replay()
        return self._out

    def __call__(self, *args):
        return _clone(self.replay(*args))
