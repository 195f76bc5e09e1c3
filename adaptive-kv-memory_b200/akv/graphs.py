"""CUDA-graph capture of a serving step's warm-tier calls.

A decode step of a serving loop runs the same layers over the same buffers
every time: per layer one ``mixed_tier_decode_attention`` (decode kernel +
LSE combine), plus the host<->device copies of the step's queries and
outputs.  Issued one by one from Python, each layer costs ~15 us of host
work (argument checks, split planning, ctypes marshalling, two launches),
which shows once the device work per layer is small (a KV-head shard on 8
GPUs runs a layer in ~30 us).  ``DecodeGraph`` records such a step once and
replays it as a single graph launch: the kernels, their split plans and
workspace are fixed at capture time, and every pointer the step reads
(queries, tiers, outputs, pinned host buffers) must stay where it was.

The decode path is capture-safe: it allocates nothing after its first call
(the split-partial workspace is cached per device and outputs may be passed
in), never synchronises, and its only host decision (the split plan)
depends on shapes alone.  The warm tier's length is baked into the graph:
recapture after tokens are appended or demoted, or pass per-row lengths
(``hot_len`` / ``warm_len`` device tensors), which the kernel reads at run
time.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch


class DecodeGraph:
    """Capture ``step()`` (any sequence of akv calls and torch copies on the
    current stream, including work forked onto other streams and joined
    back) into one CUDA graph; ``replay()`` re-issues it.

    ``warmup`` eager runs on a side stream come first, so the calls allocate
    their cached workspaces outside the capture.
    """

    def __init__(self, step: Callable[[], None], warmup: int = 2, device: Optional[torch.device] = None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                step()
        torch.cuda.current_stream(self.device).wait_stream(side)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            step()
        torch.cuda.synchronize(self.device)

    def replay(self) -> None:
        """Launch the captured step on the current stream."""
        self.graph.replay()

    def reset(self) -> None:
        """Release the graph (and the memory pool its captured allocations use)."""
        self.graph.reset()
