"""CUDA graphs of training steps on the ``xdna`` device.

A step of small layers is bound by the host: every aten call costs a few
microseconds of dispatch, and a style-transfer step makes hundreds of them.
Captured once into a CUDA graph the step replays as one launch and runs at
the speed of its kernels.  The reference has no counterpart (its NPU path is
driven from the host call by call); the capture is torch's own
(``torch.cuda.CUDAGraph``), and this module adds what the ``xdna`` allocator
needs for it: while the capture runs, xdna allocations on the capturing
stream come from a private pool that stays reserved for the graph's replays
(ATen's own allocations inside the capture go to torch's graph pool as
usual).

Rules are those of any CUDA graph: the captured function reads its inputs
from tensors that stay in place (copy fresh data into them before each
replay), makes no host synchronization and no host-to-device copy from
pageable memory, and an optimizer stepped inside the capture must be built
with ``capturable=True``.
"""
from __future__ import annotations

import contextlib
import weakref

import torch

from . import device as _device


class XdnaGraph:
    """A captured region: a ``torch.cuda.CUDAGraph`` plus the xdna memory pool
    its replays write."""

    def __init__(self):
        self.cuda_graph = torch.cuda.CUDAGraph()
        self.pool_id = 0
        self._finalizer = None

    def replay(self) -> None:
        self.cuda_graph.replay()

    def pool(self) -> int:
        """The xdna pool id, to share with another capture (``graph(..., pool=)``)."""
        return self.pool_id

    def reset(self) -> None:
        """Drop the graph and give its pool back to the allocator (tensors
        created during the capture keep their memory until they are freed)."""
        self.cuda_graph.reset()
        if self._finalizer is not None:
            self._finalizer()
            self._finalizer = None


@contextlib.contextmanager
def graph(g: XdnaGraph, pool: int = 0, stream: torch.cuda.Stream | None = None,
          capture_error_mode: str = "global"):
    """Capture the body into ``g`` (the xdna counterpart of ``torch.cuda.graph``).

    ``pool``: an xdna pool id of an earlier capture to allocate from (captures
    that replay in the order they were captured may share one)."""
    native = _device._load_native()
    with torch.cuda.graph(g.cuda_graph, stream=stream, capture_error_mode=capture_error_mode):
        s = torch.cuda.current_stream()
        g.pool_id = native.graph_capture_begin(s.device_index, s.cuda_stream, int(pool))
        if g._finalizer is None:  # the pool goes back with the graph, also after a failed capture
            g._finalizer = weakref.finalize(g, native.graph_pool_release, g.pool_id)
        try:
            yield g
        finally:
            native.graph_capture_end(s.cuda_stream)


def _detached(out):
    if isinstance(out, torch.Tensor):
        return out.detach()
    if isinstance(out, (list, tuple)):
        return type(out)(_detached(o) for o in out)
    if isinstance(out, dict):
        return {k: _detached(v) for k, v in out.items()}
    return out


def make_graphed_step(step, warmup: int = 3):
    """Warm ``step`` up on a side stream, capture one call of it, and return a
    function that replays the capture and returns what the captured call
    returned (the same tensors, detached, refreshed by every replay).

    Warm-up runs real steps (an optimizer inside ``step`` updates the weights
    ``warmup`` times before the first replay; the capture itself runs
    nothing); deferred weight gradients, autograd and the optimizer's kernels
    are all recorded in the order the eager step issues them."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(warmup):
            step()
    torch.cuda.current_stream().wait_stream(side)
    g = XdnaGraph()
    with graph(g):
        out = step()
    # the captured call's outputs are returned detached: a loss that kept its
    # autograd graph would keep that step's AccumulateGrad nodes (and the
    # stream they were created on) alive into later captures and steps
    out = _detached(out)

    def replay():
        g.replay()
        return out

    replay.graph = g
    return replay
