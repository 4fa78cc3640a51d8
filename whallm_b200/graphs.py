"""CUDA-graph capture of a whole MoE-layer forward for a fixed decode shape.

A decode step launches four to seven small kernels per layer (router logits
and top-k, then the expert call: up to a permute, a token split or gather,
the two projections and a combine, fewer for small calls); at batch 1 the GPU
work is tens of microseconds, comparable to the host cost of issuing it.  ``CapturedLayer`` records the launches once and replays them
with a single graph launch; inputs are copied into a static buffer first.
The captured kernels, streams and workspaces are the same as the eager path.
"""
from __future__ import annotations

import torch


class CapturedLayer:
    """``CapturedLayer(layer, x_example)(x) -> layer(x)`` through one graph replay.

    ``x`` must have ``x_example``'s shape and dtype.  The returned tensor is the
    graph's static output buffer (overwritten by the next replay)."""

    def __init__(self, layer, x_example: torch.Tensor, warmup: int = 2):
        self.layer = layer
        self.x = x_example.detach().clone()
        side = torch.cuda.Stream(device=self.x.device)
        side.wait_stream(torch.cuda.current_stream(self.x.device))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                layer(self.x)
        torch.cuda.current_stream(self.x.device).wait_stream(side)
        torch.cuda.synchronize(self.x.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = layer(self.x)

    def __call__(self, x: torch.Tensor | None = None) -> torch.Tensor:
        if x is not None:
            self.stage(x)
        return self.replay()

    def stage(self, x: torch.Tensor) -> None:
        """Copy ``x`` (e.g. pinned host memory) into the graph's input buffer on the
        current stream, so that a caller can stage the next input on a copy stream
        while an earlier replay runs; order the replay after it with an event."""
        if x.shape != self.x.shape or x.dtype != self.x.dtype:
            raise ValueError("captured layer expects the capture shape and dtype")
        self.x.copy_(x, non_blocking=True)

    def replay(self) -> torch.Tensor:
        """Replay on the current stream with the staged input; returns the static output."""
        self.graph.replay()
        return self.out
