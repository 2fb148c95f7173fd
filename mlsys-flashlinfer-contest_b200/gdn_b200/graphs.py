"""CUDA-graph forms of the decode step for serving loops.

A decode step of a small batch is host-bound: the kernel runs a few microseconds,
while checking and launching it from Python costs more.  A serving loop that keeps
its per-step tensors in fixed device buffers can capture the step once and replay
it: one graph launch per step, no argument checks, no allocation.  Everything the
C ABI does on the host (argument checks, grid choice) happens at capture time; the
kernels themselves are stream-ordered and allocation-free, so they capture as is.

``DecodeGraph`` captures two graphs, the state ping-ponging between two buffers
(``gdn_decode`` is out of place), or one in-place graph with ``inplace=True``.
"""
from __future__ import annotations

import torch

from . import decode


class DecodeGraph:
    """Replayable decode step over fixed buffers.

    ``q, k, v, a, b`` are the step's input buffers (fill them, then ``step()``);
    ``output`` receives o; ``state`` is the current state after every step.  The
    buffers are the caller's tensors (any valid decode arguments), captured as
    they are: refill them in place, never rebind them."""

    def __init__(self, q, k, v, state, A_log, a, dt_bias, b, scale, inplace: bool = False,
                 warmup: int = 2):
        self.q, self.k, self.v, self.a, self.b = q, k, v, a, b
        self.A_log, self.dt_bias, self.scale = A_log, dt_bias, scale
        self.output = torch.empty_like(v)
        self.inplace = inplace
        self._bufs = [state] if inplace else [state, torch.empty_like(state)]
        self._cur = 0
        self.graphs = []
        init = state.clone()
        s = torch.cuda.Stream(q.device)
        s.wait_stream(torch.cuda.current_stream(q.device))
        with torch.cuda.stream(s):
            for i in range(len(self._bufs)):  # warm up (and run the one-time setup) uncaptured
                for _ in range(warmup):
                    self._launch(i)
        torch.cuda.current_stream(q.device).wait_stream(s)
        torch.cuda.synchronize(q.device)
        self._bufs[0].copy_(init)  # the warm-up advanced the state: restore it
        for i in range(len(self._bufs)):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self._launch(i)
            self.graphs.append(g)

    def _launch(self, i):
        src = self._bufs[i]
        dst = src if self.inplace else self._bufs[1 - i]
        decode.launch(self.q, self.k, self.v, src, self.A_log, self.a, self.dt_bias, self.b,
                      self.scale, self.output, dst)

    @property
    def state(self) -> torch.Tensor:
        return self._bufs[self._cur]

    def reset_state(self, state: torch.Tensor) -> None:
        """Copy ``state`` into the current state buffer (stream-ordered)."""
        self._bufs[self._cur].copy_(state)

    def step(self) -> torch.Tensor:
        """One decode step on the current stream; returns the output buffer."""
        self.graphs[self._cur].replay()
        if not self.inplace:
            self._cur = 1 - self._cur
        return self.output
