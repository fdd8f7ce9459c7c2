"""One training step of the block stack captured in a CUDA graph.

An eager step of the 28-layer stack issues about a thousand launches from Python (the library ops,
cuBLAS GEMMs, autograd's gradient adds and, on several ranks, the bucketed NCCL all-reduces).  When a
rank's share of the batch is small, the host cannot issue them as fast as the GPU runs them.
Capturing the step once and replaying the graph removes the host from the step: forward, backward,
the gradient all-reduces (launched by the layer hooks of `LayerBucketAllReduce` during capture) and
the loss all run from one `cudaGraphLaunch`.

  step = GraphedTrainStep(model, reducer, world, loss_fn, x_example)
  loss = step(x)          # copies x into the captured input buffer, replays; returns the loss tensor

The captured step reads its input from `step.static_x` and leaves the loss in `step.static_loss` and
the global-batch gradients in the reducer's flat buffers (the parameters' .grad views).  Every rank
must capture and replay the same steps in the same order; release the step (`close()`) before the
process group is destroyed, since its graph holds NCCL work.
"""
from __future__ import annotations

import torch
import torch.distributed

from .grad_sync import LayerBucketAllReduce, train_step


class GraphedTrainStep:
    def __init__(self, model, reducer: LayerBucketAllReduce, world: int, loss_fn, x_example: torch.Tensor,
                 warmup: int = 3, pool=None, allreduce: bool = True):
        self.model, self.reducer, self.world, self.loss_fn = model, reducer, world, loss_fn
        self.static_x = x_example.detach().clone()
        saved_world = reducer.world
        if not allreduce:                # a compute-only step (no collective), e.g. to time the comm
            reducer.world = 1
        try:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):        # warm-up: cuBLAS handles, NCCL channels, allocator
                for _ in range(warmup):
                    train_step(model, self.static_x, reducer, world, loss_fn)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            # With a process group, the NCCL watchdog thread keeps querying events of earlier
            # collectives while this thread captures: restrict the capture checks to this thread.
            mode = "thread_local" if torch.distributed.is_initialized() else "global"
            with torch.cuda.graph(self.graph, pool=pool, capture_error_mode=mode):
                self.static_loss = train_step(model, self.static_x, reducer, world, loss_fn)
            torch.cuda.synchronize()
        finally:
            reducer.world = saved_world

    def pool(self):
        return self.graph.pool()

    def __call__(self, x: torch.Tensor | None = None) -> torch.Tensor:
        if x is not None:
            self.static_x.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.static_loss

    def close(self):
        if getattr(self, "graph", None) is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None
