"""CUDA-graph replay of a forward built on this package's operators.

Every launch of the library goes to the current stream with its arguments by value
(tensor maps included), workspaces come from torch's caching allocator and nothing
synchronises the host, so a forward such as ``TransformerLM`` prefill can be
captured once and replayed: one graph launch instead of tens of kernel launches and
their Python overhead per call.
"""

from __future__ import annotations

from typing import Callable

import torch


class CapturedForward:
    """``fn(*args)`` captured into a CUDA graph on static input buffers.

    ``__call__(*args)`` copies the new inputs into the static buffers, replays the
    graph on the current stream and returns the static output (overwritten by the
    next call: clone it to keep it).  Shapes, dtypes and devices are fixed by the
    example arguments.
    """

    def __init__(self, fn: Callable, *example_args: torch.Tensor, warmup: int = 2):
        self.fn = fn
        self.static_args = [a.clone() for a in example_args]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(warmup):  # first calls set up workspaces, weights caches and kernel attributes
                fn(*self.static_args)
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.static_out = fn(*self.static_args)

    def __call__(self, *args: torch.Tensor):
        if len(args) != len(self.static_args):
            raise ValueError(f"expected {len(self.static_args)} inputs, got {len(args)}")
        for dst, src in zip(self.static_args, args):
            if src.shape != dst.shape or src.dtype != dst.dtype:
                raise ValueError(f"input {tuple(src.shape)} {src.dtype} does not match the captured "
                                 f"{tuple(dst.shape)} {dst.dtype}")
            dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.static_out
