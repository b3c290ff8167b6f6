"""CUDA-graph capture of a denoise step (the block loop of
LTX_2_MLX/model/model.py:1044-1310, ``_process_transformer_blocks``).

A step is ~50 library launches and ~40 torch launches per block, ~4300 for
the 48-block 22B model.  Eagerly, each costs host time (Python, ctypes,
tensor-map encoding, launch); on a few GPUs the device work per block is
small enough for that to show.  ``StepGraph`` captures the whole step once
and replays it: inputs are read from the tensors the step was captured with,
so callers copy new inputs into ``static_args`` before ``replay()``.

Every library entry point is capture-safe: no host synchronization, no
allocation outside torch's caching allocator (which gives the graph its own
pool), tensor maps encoded on the host at capture time and baked into the
kernel parameters.  NCCL collectives (the K/V all-gathers of a row-sharded
step) are captured as well; every rank must capture the same step.
"""

from __future__ import annotations

import torch

from . import _lib


class StepGraph:
    """``fn(*static_args)`` captured in one CUDA graph.

    ``warmup`` eager calls run first on a side stream (as torch requires
    before capture).  ``launches`` is the number of library kernels the
    captured step launches per replay."""

    def __init__(self, fn, *static_args, warmup: int = 1):
        self.fn = fn
        self.static_args = static_args
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn(*static_args)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        n0 = _lib.launch_count()
        # thread_local: the NCCL watchdog thread may query events meanwhile
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            self.out = fn(*static_args)
        self.launches = _lib.launch_count() - n0

    def replay(self):
        """Re-run the captured step on the current stream; returns the
        captured outputs (overwritten in place)."""
        self.graph.replay()
        return self.out

    def release(self) -> None:
        """Free the graph (before destroying a process group whose
        collectives it holds)."""
        self.graph.reset()
        self.graph = None
        self.out = None
