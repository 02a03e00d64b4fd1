"""CUDA-graph replay of a layer call on static buffers.

Small layers (hidden 256, T = 1024) and single-token
decode steps are launch-bound: the layer issues about twenty kernels
(projection GEMMs, the activation pass, the recurrence, o_proj), each a few
microseconds of work.  ``GraphedCall`` captures one call into a CUDA graph and
replays it, so a step costs one graph launch.

The captured call must be free of host synchronisation and must read its
inputs from, and write its outputs to, the same device tensors on every
replay: copy new inputs into ``static_inputs`` before ``replay()``; the
returned tensor is the same object each time (the layer's state, when the call
carries one, is updated in place by every replay).  Everything the library
launches is capturable: its kernels take the caller's stream and it allocates
no device memory itself (workspaces come from torch's caching allocator, which
keeps them alive with the graph's memory pool).
"""
from __future__ import annotations

import torch


class GraphedCall:
    """fn(*static_inputs) captured once; ``replay()`` re-runs it."""

    def __init__(self, fn, *static_inputs, warmup: int = 2):
        self.fn = fn
        self.static_inputs = static_inputs
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # warm-up outside the capture: library set-up, allocator pools
            for _ in range(max(1, warmup)):
                fn(*static_inputs)
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.output = fn(*static_inputs)

    def replay(self):
        """Run the captured call again on the current stream; returns the static output."""
        self.graph.replay()
        return self.output
