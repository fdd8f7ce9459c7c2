"""Per-call dispatch between the eager and the compile path (same rule as the reference's
library/_compat.py:1-8).

- Under torch.compile the public functions call the registered operator (krsi::*_fwd), which
  the compiler traces as one opaque node with a fake implementation and registered autograd
  (see _ext.py), so fullgraph=True and torch.export work.
- In eager they call a plain torch.autograd.Function that invokes the same operators. The
  operators are C++ registrations, so the eager path costs one dispatcher call per op.
"""
import torch


def compiling() -> bool:
    return torch.compiler.is_compiling()
