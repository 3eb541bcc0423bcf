"""Fixed-shape MoE forwards replayed from one CUDA graph.

The reference's decode loop (generate.rs:811-880, driven through CausalLM::forward,
generate.rs:280-287) runs the same per-token work every step; on the B200 its MoE part
(one block, a decoder layer's FFN half, or the whole stack of them) is captured once and
replayed as a single graph launch per step, so a step costs no host launch work beyond
the input copy. Every kernel of the block is graph-safe: scratch is sized by a warm-up
call before the capture and nothing is allocated or synchronised inside it.
"""
from __future__ import annotations

from typing import Callable

import torch


class GraphedForward:
    """``fn(x) -> y`` for x of one fixed shape, replayed from a CUDA graph.

    ``g = GraphedForward(stack, x_example)``; ``y = g(x)`` copies x into the graph's
    input buffer, replays, and returns the graph's output buffer (overwritten by the
    next call: copy it to keep it)."""

    def __init__(self, fn: Callable[[torch.Tensor], torch.Tensor], example: torch.Tensor, warmup: int = 2):
        if not example.is_cuda:
            raise ValueError("GraphedForward needs a CUDA tensor")
        self.fn = fn
        self.device = example.device
        self.static_x = example.detach().clone()
        cur = torch.cuda.current_stream(self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):  # sizes every context's scratch, sets kernel attributes
            for _ in range(max(1, warmup)):
                fn(self.static_x)
        cur.wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.static_y = fn(self.static_x)
        torch.cuda.synchronize(self.device)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape != self.static_x.shape or x.dtype != self.static_x.dtype:
            raise ValueError(f"captured for {tuple(self.static_x.shape)} {self.static_x.dtype}, "
                             f"got {tuple(x.shape)} {x.dtype}")
        self.static_x.copy_(x)
        self.graph.replay()
        return self.static_y

    def replay(self) -> torch.Tensor:
        """Replay on whatever the input buffer ``static_x`` holds."""
        self.graph.replay()
        return self.static_y


__all__ = ["GraphedForward"]
