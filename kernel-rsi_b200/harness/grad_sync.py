"""Weight-gradient all-reduce for the batch-sharded block harness.

Each rank runs forward+backward on its own batch shard; the only collective is one SUM all-reduce
per bucket of weight gradients (the loss is pre-scaled by 1/world, so the sum is the global-batch
gradient).  Gradients live in one flat buffer per bucket (param.grad are views into it), so no
packing copies are needed, and a bucket is launched asynchronously (NCCL's own stream) the moment
autograd has accumulated its last gradient, so its communication overlaps the rest of the backward.

Buckets: the bf16 weights of `layers_per_bucket` consecutive layers (backward order: the last
layers' bucket fills first), except the first `tail_layers` layers, which get one bucket each (the
final buckets' all-reduces cannot overlap any backward work, so they are kept small), and the small
fp32 tensors of every layer (the relative-position tables, 131 KB a layer) in one bucket of their
own, launched when the first layer's table gradient lands near the end of the backward (one
collective instead of one latency-bound call per layer).
"""
from __future__ import annotations

from collections import defaultdict

import torch
import torch.distributed as dist


class LayerBucketAllReduce:
    def __init__(self, layers, group=None, layers_per_bucket: int = 1, small_bytes: int = 1 << 20,
                 tail_layers: int = 0):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.buckets = []       # (bucket key, dtype, flat buffer, [params])
        self.pending = defaultdict(int)
        self.ready = set()
        self.handles = []
        self.param_bucket = {}
        n = len(layers)
        groups = defaultdict(list)      # key -> params, in layer order
        per_layer_bytes = defaultdict(int)   # the largest layer's share of each dtype
        for li, layer in enumerate(layers):
            by_dtype = defaultdict(int)
            for p in layer.parameters():
                if p.requires_grad:
                    by_dtype[p.dtype] += p.numel() * p.element_size()
            for dt, b in by_dtype.items():
                per_layer_bytes[dt] = max(per_layer_bytes[dt], b)
        direct = set()          # weights whose GEMM backward writes the bucket slot itself
        for li, layer in enumerate(layers):
            lw = getattr(layer, "linear_weights", None)
            direct.update(lw() if lw is not None else [])
            for p in layer.parameters():
                if not p.requires_grad:
                    continue
                if per_layer_bytes[p.dtype] < small_bytes:
                    key = ("all", p.dtype)                              # one bucket for all layers
                elif li < tail_layers:
                    key = (("tail", li), p.dtype)                       # the last layers: one bucket each
                else:
                    key = ((n - 1 - li) // max(1, layers_per_bucket), p.dtype)
                groups[key].append(p)
        from .block import set_grad_sink

        self.zero_tails = []    # the accumulated (not directly written) part of each bucket
        for key, params in groups.items():
            params = [p for p in params if p in direct] + [p for p in params if p not in direct]
            total = sum(p.numel() for p in params)
            flat = torch.zeros(total, dtype=params[0].dtype, device=params[0].device)
            off = 0
            for p in params:
                p.grad = flat[off: off + p.numel()].view_as(p)
                off += p.numel()
                self.param_bucket[p] = len(self.buckets)
                if p in direct:
                    set_grad_sink(p, self)
            n_direct = sum(p.numel() for p in params if p in direct)
            if n_direct < total:
                self.zero_tails.append(flat[n_direct:])
            self.buckets.append((key, params[0].dtype, flat, params))
        # direct weights normally bypass autograd's accumulation (so their hook never fires); if one
        # is ever handed to autograd instead, its hook still marks it ready exactly once
        self.hooks = [p.register_post_accumulate_grad_hook(self.mark_ready) for p in self.param_bucket]

    @property
    def bytes(self) -> int:
        return sum(f.numel() * f.element_size() for _, _, f, _ in self.buckets)

    def zero_grad(self):
        """Zero the slots that autograd accumulates into; the GEMM weights' slots are overwritten
        by their backward."""
        for tail in self.zero_tails:
            tail.zero_()
        self.pending.clear()
        self.ready.clear()
        self.handles.clear()

    def mark_ready(self, p):
        """Gradient of p is final for this step; launches its bucket's all-reduce when complete.
        Repeated calls for one parameter in a step count once (autograd may still run the
        accumulate hook of a weight whose GEMM backward wrote its gradient itself)."""
        if id(p) in self.ready:
            return
        self.ready.add(id(p))
        bi = self.param_bucket[p]
        self.pending[bi] += 1
        _, _, flat, params = self.buckets[bi]
        if self.pending[bi] == len(params) and self.world > 1:
            self.handles.append(dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True))

    def wait(self):
        """Make the current stream wait for every launched all-reduce (no host sync)."""
        for h in self.handles:
            h.wait()
        self.handles.clear()

    def remove(self):
        from .block import clear_grad_sink

        for h in self.hooks:
            h.remove()
        for p in self.param_bucket:
            clear_grad_sink(p, self)


def shard_batch(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank r's contiguous slice of the global batch (equal shards; B divisible by world)."""
    B = x.shape[0]
    if B % world:
        raise ValueError(f"global batch {B} is not divisible by world size {world}")
    n = B // world
    return x[rank * n: (rank + 1) * n]


def train_step(model, x_local, reducer: LayerBucketAllReduce, world: int, loss_fn):
    """Forward + backward on this rank's shard; returns the global-mean loss contribution of this
    rank (loss_local / world) as a device tensor.  Gradients end as the global-batch gradient."""
    reducer.zero_grad()
    out = model(x_local)
    loss = loss_fn(out) / world
    loss.backward()
    reducer.wait()
    return loss.detach()
