"""The 28-layer pre-norm block stack of BASELINE config 5, built on the drop-in library ops.

Each layer:  x -> RMSNorm -> fused q|k|v GEMM -> relpos attention (H heads of D) -> out GEMM + x
                -> RMSNorm -> merged gate|value GEMM (d -> 2F) -> GEGLU -> down GEMM (F -> d) + x
(the residual adds ride in the out and down GEMMs: addmm with beta = 1; the weight gradients of
the four GEMMs are written straight into the all-reduce buckets when a LayerBucketAllReduce owns
them)
The attention, RMSNorm and GEGLU calls are the kernel-rsi library functions (relpos_attention(),
rmsnorm(), geglu(), with the reference's signatures); the GEMMs are torch matmuls (cuBLAS), except
that on the B200 kernels the gate|value GEMM and the GEGLU forward are one tcgen05 kernel
(krsi::linear_geglu_fwd, GEGLU in the GEMM's epilogue) and so are the down projection's input
gradient and GEGLU's backward (krsi::linear_geglu_bwd).  loss = mean(out.float()^2).  Weights are
bf16 ~ N(0, 0.02) (RMSNorm weights 1 + N(0, 0.02)), the per-layer relative-position table pd
[H, 2L-1] is fp32 ~ N(0, 0.02).

`ops` supplies the three library functions, so the same model runs on the B200 kernels or, for
CPU tests of the distributed harness, on any stand-in with the same signatures.
"""
from __future__ import annotations

import math
import weakref
from dataclasses import dataclass

import torch
from torch import nn

# id(weight) -> (weak weight, weak bucket owner): the gradient all-reduce that owns the weight's
# .grad slot (see _Linear).  Keyed by identity and held weakly, so copies of a model (deepcopy makes
# new Parameters) and dropped reducers leave no trace.
_GRAD_SINKS: dict = {}


def set_grad_sink(w: torch.Tensor, owner) -> None:
    _GRAD_SINKS[id(w)] = (weakref.ref(w), weakref.ref(owner))


def clear_grad_sink(w: torch.Tensor, owner) -> None:
    if grad_sink(w) is owner:
        del _GRAD_SINKS[id(w)]


def grad_sink(w: torch.Tensor):
    entry = _GRAD_SINKS.get(id(w))
    if entry is None or entry[0]() is not w:
        return None
    return entry[1]()


class _Linear(torch.autograd.Function):
    """y = x @ w^T (+ res, with beta = 1).  When the weight's gradient lives in a bucket of a
    gradient all-reduce (grad_sink(w), set by LayerBucketAllReduce), the backward writes
    dW = g^T x straight into the weight's .grad view of the bucket (cuBLAS with `out=`) and tells
    the bucket it is ready, instead of handing dW to autograd, which would add it onto a zeroed
    bucket: a zero pass and a read-modify-write of every weight gradient each step."""

    @staticmethod
    def forward(ctx, x, w, res):
        ctx.save_for_backward(x, w)
        ctx.w = w
        ctx.has_res = res is not None
        return torch.addmm(res, x, w.t()) if res is not None else x @ w.t()

    @staticmethod
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        gx = g @ w if ctx.needs_input_grad[0] else None
        gw = _weight_grad(ctx.w, g, x) if ctx.needs_input_grad[1] else None
        return gx, gw, (g if ctx.has_res else None)


@dataclass
class BlockConfig:
    layers: int = 28
    d: int = 1152
    heads: int = 16
    head_dim: int = 72
    ffn: int = 4608
    seq: int = 1024
    eps: float = 1e-6

    def params_per_layer(self) -> int:
        return 3 * self.d * self.d + self.d * self.d + 2 * self.ffn * self.d + self.ffn * self.d

    def linear_params(self) -> int:
        return self.layers * self.params_per_layer()

    def flops_per_token(self) -> int:
        """Training FLOPs per token: 6 x linear params (GEMMs) + 12 x L x H x D x layers (attention,
        fwd 4 + bwd 8 per query per key, D unpadded)."""
        return 6 * self.linear_params() + 12 * self.seq * self.heads * self.head_dim * self.layers


class _RMSNormSkip(torch.autograd.Function):
    """(rmsnorm(x, w, eps), x) for a pre-norm residual block, where x feeds both the norm and the
    residual branch: the backward gets both gradients of x at once and adds them inside the RMSNorm
    backward kernel (krsi::rmsnorm_bwd_add) instead of in a separate autograd pass over x."""

    @staticmethod
    def forward(ctx, x2d, w, eps):
        y, rstd = torch.ops.krsi.rmsnorm_fwd(x2d, w, eps)
        ctx.save_for_backward(x2d, w, rstd)
        return y, x2d.view_as(x2d)

    @staticmethod
    def backward(ctx, gy, gskip):
        x2d, w, rstd = ctx.saved_tensors
        if gy is None:
            return gskip, None, None
        if gskip is None:
            dx, dw = torch.ops.krsi.rmsnorm_bwd(gy.contiguous(), x2d, w, rstd)
        else:
            dx, dw = torch.ops.krsi.rmsnorm_bwd_add(gy.contiguous(), x2d, w, rstd, gskip.contiguous())
        return dx, dw, None


def _weight_grad(w, g, x):
    """dW = g^T x: written straight into the weight's bucket view when a gradient all-reduce owns it
    (and the bucket told it is ready), else returned for autograd to accumulate."""
    sink = grad_sink(w)
    if sink is not None and w.grad is not None:
        torch.mm(g.t(), x, out=w.grad)
        sink.mark_ready(w)
        return None
    return g.t() @ x


class _FeedForward(torch.autograd.Function):
    """res + geglu(x @ wi^T) @ wo^T on the two fused kernels: the gate|value projection with GEGLU in
    its epilogue (krsi::linear_geglu_fwd, which also returns u) and, in the backward, the down
    projection's input gradient with GEGLU's backward in its epilogue (krsi::linear_geglu_bwd), so
    GEGLU's input gradient never reaches memory.  Weight gradients go into their buckets as in
    _Linear."""

    @staticmethod
    def forward(ctx, x, wi, wo, res, ops):
        u, g = ops.linear_geglu_fwd(x, wi)
        ctx.save_for_backward(x, wi, wo, u, g)
        ctx.wi, ctx.wo, ctx.ops = wi, wo, ops
        return torch.addmm(res, g, wo.t())

    @staticmethod
    def backward(ctx, gy):
        x, wi, wo, u, g = ctx.saved_tensors
        gy = gy.contiguous()
        gwo = _weight_grad(ctx.wo, gy, g) if ctx.needs_input_grad[2] else None
        du = ctx.ops.linear_geglu_bwd(gy, wo, u)
        gx = du @ wi if ctx.needs_input_grad[0] else None
        gwi = _weight_grad(ctx.wi, du, x) if ctx.needs_input_grad[1] else None
        return gx, gwi, gwo, gy, None


def _feed_forward(ops, h, wi, wo, res):
    """res + geglu(h @ wi^T) @ wo^T: the fused kernels when `ops` runs on the B200 kernels."""
    if getattr(ops, "fused_ffn", False):
        return _FeedForward.apply(h, wi, wo, res, ops)
    return _Linear.apply(ops.geglu(_Linear.apply(h, wi, None)), wo, res)


def _norm_and_skip(ops, x2, w, eps):
    """The normalised rows and the residual input: fused when `ops` runs on the B200 kernels."""
    if getattr(ops, "fused_norm_skip", False):
        return _RMSNormSkip.apply(x2, w, eps)
    return ops.rmsnorm(x2, w, eps), x2


class Layer(nn.Module):
    def __init__(self, cfg: BlockConfig, ops, gen: torch.Generator, device, dtype=torch.bfloat16):
        super().__init__()
        self.cfg, self.ops = cfg, ops
        d, F_, H = cfg.d, cfg.ffn, cfg.heads

        def w(*shape, std=0.02, mean=0.0):
            t = torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std + mean
            return nn.Parameter(t.to(dtype))

        self.norm1 = w(d, mean=1.0)
        self.wqkv = w(3 * d, d)
        self.wo = w(d, d)
        self.norm2 = w(d, mean=1.0)
        self.wi = w(2 * F_, d)          # rows [0, F) gate, [F, 2F) value
        self.wo2 = w(d, F_)
        self.pd = nn.Parameter(torch.randn(H, 2 * cfg.seq - 1, generator=gen, device=device) * 0.02)

        self.attn_marks = None          # optional AttentionTimer events (forward and backward)

    def forward(self, x):
        cfg, ops = self.cfg, self.ops
        B, L, d = x.shape
        x2 = x.reshape(B * L, d)
        h, x2 = _norm_and_skip(ops, x2, self.norm1, cfg.eps)
        qkv = _Linear.apply(h, self.wqkv, None)
        marks = self.attn_marks
        if marks is not None:           # fwd begin / bwd end
            qkv = _Mark.apply(qkv, marks[0], marks[3])
        a = ops.relpos_attention(qkv, self.pd, B, L, cfg.heads, cfg.head_dim, 1.0 / math.sqrt(cfg.head_dim))
        if marks is not None:           # fwd end / bwd begin
            a = _Mark.apply(a, marks[1], marks[2])
        x2 = _Linear.apply(a, self.wo, x2)          # residual add inside the GEMM (beta = 1)
        h, x2 = _norm_and_skip(ops, x2, self.norm2, cfg.eps)
        x2 = _feed_forward(ops, h, self.wi, self.wo2, x2)
        return x2.reshape(B, L, d)

    def linear_weights(self):
        """The weights used through _Linear / _FeedForward (their gradients can be written into a
        bucket)."""
        return [self.wqkv, self.wo, self.wi, self.wo2]


class _Mark(torch.autograd.Function):
    """Identity on a tensor that records one CUDA event when the forward passes it and another
    when its gradient passes back; placed on either side of an op it brackets the op's forward and
    backward kernels on the stream without touching the op itself."""

    @staticmethod
    def forward(ctx, x, fwd_event, bwd_event):
        if fwd_event is not None:
            fwd_event.record()
        ctx.bwd_event = bwd_event
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        if ctx.bwd_event is not None:
            ctx.bwd_event.record()
        return g, None, None


class AttentionTimer:
    """CUDA events around every layer's attention forward and backward.  The events are created
    `external`, so they keep timing when the step is captured in a CUDA graph; read them after the
    step (or the replay) has completed."""

    def __init__(self, stack: "BlockStack"):
        mk = lambda: torch.cuda.Event(enable_timing=True, external=True)  # noqa: E731
        self.marks = []
        for layer in stack.layers:
            m = (mk(), mk(), mk(), mk())     # fwd begin, fwd end, bwd begin, bwd end
            layer.attn_marks = m
            self.marks.append(m)

    def fwd_ms(self) -> float:
        return sum(a.elapsed_time(b) for a, b, _, _ in self.marks)

    def bwd_ms(self) -> float:
        return sum(c.elapsed_time(d) for _, _, c, d in self.marks)


class BlockStack(nn.Module):
    def __init__(self, cfg: BlockConfig, ops, device, seed: int = 0, dtype=torch.bfloat16):
        super().__init__()
        self.cfg = cfg
        gen = torch.Generator(device=device).manual_seed(seed)
        self.layers = nn.ModuleList(Layer(cfg, ops, gen, device, dtype) for _ in range(cfg.layers))

    def forward(self, x):
        for layer in self.layers:
            x = layer(x)
        return x


def loss_fn(out: torch.Tensor) -> torch.Tensor:
    return out.float().pow(2).mean()


class LibraryOps:
    """The kernel-rsi library functions (B200 kernels); imported lazily so CPU-only users of the
    harness need not load the native extension."""

    def __init__(self):
        import geglu
        import relpos_attention
        import rmsnorm

        self.rmsnorm = rmsnorm.rmsnorm
        self.geglu = geglu.geglu
        self.relpos_attention = relpos_attention.relpos_attention
        # RMSNorm and the residual branch share their input: one backward kernel adds both gradients
        self.fused_norm_skip = True
        # the feed-forward on the fused kernels: the gate|value projection with GEGLU in its epilogue,
        # the down projection's input gradient with GEGLU's backward in its epilogue
        import linear_geglu  # noqa: F401  (loads the library's op registrations)
        self.linear_geglu_fwd = torch.ops.krsi.linear_geglu_fwd
        self.linear_geglu_bwd = torch.ops.krsi.linear_geglu_bwd
        self.fused_ffn = True
