"""The block stack at its real dims on the GPU, against the reference path.

Two layers of d=1152, H=16, D=72, F=4608, L=1024, B=2, built on the library ops (LibraryOps: the
B200 kernels), are checked against the same bf16 weights run in fp32 through the reference's own
eager expressions (rmsnorm/geglu/relpos_attention `reference()`, SDPA on the math backend, TF32
off), as the reference's tools build their fp32 run of the original (tools/common.py:476-490):
the output, the loss and every parameter gradient within 1e-2 normalised max error, and the
reference's compare() criterion against the bf16 original.  Also: the CUDA-graph step the bench
replays gives the eager step's loss and gradients; and, on two GPUs, the NCCL-averaged gradients of
the batch-sharded step equal the one-rank full-batch gradients."""
import copy
import os
import socket
import sys
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG, ROOT

sys.path.insert(0, str(PKG))

from harness.block import BlockConfig, BlockStack, LibraryOps, loss_fn  # noqa: E402
from harness.grad_sync import LayerBucketAllReduce, shard_batch, train_step  # noqa: E402
from harness.inputs import gen  # noqa: E402
from oracle import ops as O  # noqa: E402
from oracle.compare import compare, norm_max_err  # noqa: E402

pytestmark = pytest.mark.gpu
dev = "cuda"
CFG = BlockConfig(layers=2)          # the real layer dims, two layers


class RefOps:
    rmsnorm = staticmethod(O.rmsnorm_reference)
    geglu = staticmethod(O.geglu_reference)
    relpos_attention = staticmethod(O.relpos_reference)


def batch(B):
    return gen((B, CFG.seq, CFG.d), 77, torch.bfloat16)


def with_ops(model, ops, dtype=None):
    m = copy.deepcopy(model)
    for layer in m.layers:
        layer.ops = ops
    if dtype is not None:
        m = m.to(dtype)
        for layer in m.layers:            # pd is fp32 in every variant
            layer.pd.data = layer.pd.data.float()
    return m


def fwd_bwd(model, x):
    model.zero_grad(set_to_none=True)
    out = model(x)
    loss = loss_fn(out)
    loss.backward()
    names = [n for n, _ in model.named_parameters()]
    return [out.detach(), loss.detach()] + [p.grad.detach() for _, p in model.named_parameters()], names


def test_block_stack_matches_the_fp32_reference_path():
    cand_model = BlockStack(CFG, LibraryOps(), dev, seed=0)
    x = batch(2).to(dev)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref32, names = fwd_bwd(with_ops(cand_model, RefOps(), torch.float32), x.float())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    orig, _ = fwd_bwd(with_ops(cand_model, RefOps()), x)
    cand, _ = fwd_bwd(cand_model, x)
    labels = ["out", "loss"] + names
    assert len(labels) == 2 + 7 * CFG.layers
    errs = {k: norm_max_err(c.float(), r.float()) for k, c, r in zip(labels, cand, ref32)}
    bad = {k: e for k, e in errs.items() if not e <= 1e-2}
    assert not bad, bad
    res = compare([r.float() for r in ref32], [o.float() for o in orig], [c.float() for c in cand])
    assert res["pass"], [(k, o) for k, o in zip(labels, res["outputs"]) if not o.get("passed", True)]


def test_graphed_step_matches_eager_step():
    from harness.graphed import GraphedTrainStep

    model = BlockStack(CFG, LibraryOps(), dev, seed=1)
    reducer = LayerBucketAllReduce(model.layers)
    x = batch(2).to(dev)
    loss_e = train_step(model, x, reducer, 1, loss_fn).clone()
    grads_e = [p.grad.clone() for p in model.parameters()]
    step = GraphedTrainStep(model, reducer, 1, loss_fn, torch.zeros_like(x))
    try:
        loss_g = step(x).clone()
        torch.cuda.synchronize()
        grads_g = [p.grad.clone() for p in model.parameters()]
        assert abs(loss_g.item() - loss_e.item()) <= 1e-5 * abs(loss_e.item())
        for a, b in zip(grads_g, grads_e):
            assert norm_max_err(a.float(), b.float()) <= 1e-2   # dQ sums in arrival order
        # a second replay on new data reads the new input
        x2 = batch(2).to(dev).flip(0)
        loss_2 = step(x2).clone()
        assert abs(train_step(model, x2, reducer, 1, loss_fn).item() - loss_2.item()) <= 1e-5 * abs(loss_2.item())
    finally:
        step.close()


# ---------------------------------------------------------------- two GPUs, NCCL

def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(PKG))
    sys.path.insert(0, str(PKG / "library"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        from harness.graphed import GraphedTrainStep

        model = BlockStack(CFG, LibraryOps(), torch.device("cuda", rank), seed=2)
        reducer = LayerBucketAllReduce(model.layers)
        xg = batch(4)
        x = shard_batch(xg, rank, world).to(f"cuda:{rank}")
        loss = train_step(model, x, reducer, world, loss_fn)
        eager = [p.grad.float().cpu().numpy().copy() for p in model.parameters()]
        step = GraphedTrainStep(model, reducer, world, loss_fn, x)
        loss_g = step(x).clone()
        torch.cuda.synchronize()
        graphed = [p.grad.float().cpu().numpy().copy() for p in model.parameters()]
        step.close()
        q.put((rank, "ok", float(loss), float(loss_g), eager, graphed))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", f"{type(e).__name__}: {e}", None, None, None))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_allreduced_gradients_equal_full_batch():
    # the one-rank full-batch step on GPU 0 first (no process group in this process)
    model = BlockStack(CFG, LibraryOps(), dev, seed=2)
    reducer = LayerBucketAllReduce(model.layers)
    loss_full = train_step(model, batch(4).to(dev), reducer, 1, loss_fn).item()
    ref = [p.grad.float().cpu() for p in model.parameters()]
    del model, reducer
    torch.cuda.synchronize()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, status, loss, loss_g, eager, graphed = q.get(timeout=600)
        res[r] = (status, loss, loss_g, eager, graphed)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert all(v[0] == "ok" for v in res.values()), res
    assert abs(res[0][1] + res[1][1] - loss_full) <= 1e-3 * abs(loss_full)
    assert abs(res[0][2] + res[1][2] - loss_full) <= 1e-3 * abs(loss_full)
    for r in (0, 1):
        for which in (3, 4):                 # eager and graphed steps
            for g, gref in zip(res[r][which], ref):
                assert norm_max_err(torch.from_numpy(g), gref) <= 1e-2


def test_fused_ffn_matches_the_unfused_block():
    """The block with the gate|value GEMM and GEGLU as one kernel (krsi::linear_geglu_fwd) against the
    same block with cuBLAS's GEMM followed by the GEGLU kernel: the fused kernel rounds u once from an
    fp32 accumulator as cuBLAS does and applies the GEGLU kernel's arithmetic to it, so the loss, the
    output and every gradient agree to the accumulation order of the two GEMMs.  The forward is
    deterministic (output and loss to 1e-3); the gradients also carry the attention backward's
    run-to-run dQ accumulation order (its TMA reduce-adds land in any order), so they are held to
    the block's 1e-2."""
    ops = LibraryOps()
    model = BlockStack(CFG, ops, dev, seed=3)
    unfused_ops = LibraryOps()
    unfused_ops.fused_ffn = False
    x = batch(2).to(dev)
    fused, names = fwd_bwd(model, x)
    unfused, _ = fwd_bwd(with_ops(model, unfused_ops), x)
    labels = ["out", "loss"] + names
    errs = {k: norm_max_err(a.float(), b.float()) for k, a, b in zip(labels, fused, unfused)}
    bad = {k: e for k, e in errs.items() if not e <= (1e-3 if k in ("out", "loss") else 1e-2)}
    assert not bad, bad
