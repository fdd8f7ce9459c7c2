"""The batch-sharded block harness on CPU ranks (gloo): sharding, the layer-bucket gradient
all-reduce (N-rank averaged gradients == 1-rank full-batch gradients), and failure detection (a
rank that dies or never joins ends the others' collectives with an error instead of a hang).
The model runs on the oracle's reference functions (CPU stand-ins with the library signatures)."""
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


class OracleOps:
    def __init__(self):
        from oracle import ops as O
        self.rmsnorm = O.rmsnorm_reference
        self.geglu = O.geglu_reference
        self.relpos_attention = O.relpos_reference


def tiny_cfg():
    from harness.block import BlockConfig
    return BlockConfig(layers=2, d=16, heads=2, head_dim=8, ffn=24, seq=8)


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def make_model(cfg):
    from harness.block import BlockStack
    return BlockStack(cfg, OracleOps(), torch.device("cpu"), seed=3, dtype=torch.float32)


def global_batch(cfg, B=4):
    g = torch.Generator().manual_seed(9)
    return torch.randn(B, cfg.seq, cfg.d, generator=g)


def test_shard_batch():
    from harness.grad_sync import shard_batch
    x = torch.arange(8).view(8, 1)
    assert shard_batch(x, 1, 4).flatten().tolist() == [2, 3]
    with pytest.raises(ValueError):
        shard_batch(x, 0, 3)


def test_config_matches_baseline_numbers():
    from harness.block import BlockConfig
    c = BlockConfig()
    assert c.linear_params() == 594_542_592
    assert c.flops_per_token() * 32 * 1024 == 129_879_811_031_040


def _worker(rank, world, port, q, mode):
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(PKG))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
        from harness.block import loss_fn
        from harness.grad_sync import LayerBucketAllReduce, shard_batch, train_step
        cfg = tiny_cfg()
        model = make_model(cfg)
        # "ok": default buckets (this tiny model's tensors all fall in the one small-tensor bucket);
        # "per_layer": one bucket per layer and dtype; "pairs": two layers per bucket
        kw = {"per_layer": dict(small_bytes=0), "pairs": dict(small_bytes=0, layers_per_bucket=2),
              "tail": dict(small_bytes=0, layers_per_bucket=2, tail_layers=1)}.get(mode, {})
        reducer = LayerBucketAllReduce(model.layers, **kw)
        if mode == "die" and rank == 1:
            raise RuntimeError("planted failure on rank 1 before its first collective")
        x = shard_batch(global_batch(cfg), rank, world)
        loss = train_step(model, x, reducer, world, loss_fn)
        # numpy copies travel by value: a tensor would be shared through a file descriptor that
        # dies with this process if it exits before the parent has received it
        grads = {n: p.grad.detach().numpy().copy() for n, p in model.named_parameters()}
        q.put((rank, "ok", float(loss), grads))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", f"{type(e).__name__}: {e}", None))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run_ranks(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, status, val, grads = q.get(timeout=120)
        out[r] = (status, val, grads)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("mode", ["ok", "per_layer", "pairs", "tail"])
def test_two_rank_gradients_equal_full_batch(mode):
    from harness.block import loss_fn
    from harness.grad_sync import LayerBucketAllReduce, train_step
    cfg = tiny_cfg()
    model = make_model(cfg)
    reducer = LayerBucketAllReduce(model.layers)   # world 1: no collective
    loss = train_step(model, global_batch(cfg), reducer, 1, loss_fn)
    ref = {n: p.grad.clone() for n, p in model.named_parameters()}
    res = run_ranks(2, mode)
    assert all(v[0] == "ok" for v in res.values()), res
    assert abs(res[0][1] + res[1][1] - float(loss)) < 1e-5 * max(1.0, abs(float(loss)))
    for r in (0, 1):
        for n, g in res[r][2].items():
            torch.testing.assert_close(torch.from_numpy(g), ref[n], rtol=1e-4, atol=1e-6)


def test_bucket_plan():
    from harness.block import BlockConfig, BlockStack
    from harness.grad_sync import LayerBucketAllReduce

    cfg = BlockConfig(layers=4, d=64, heads=2, head_dim=32, ffn=128, seq=16)
    model = BlockStack(cfg, OracleOps(), torch.device("cpu"), seed=0, dtype=torch.bfloat16)
    red = LayerBucketAllReduce(model.layers, layers_per_bucket=2, small_bytes=1024)
    keys = [k for k, _, _, _ in red.buckets]
    # bf16 weights: layers (3, 2) and (1, 0) in backward order; the fp32 tables of all layers: one bucket
    assert sorted(k for k in keys if k[1] == torch.bfloat16) == [(0, torch.bfloat16), (1, torch.bfloat16)]
    assert (("all", torch.float32)) in keys and len(keys) == 3
    red.remove()
    red = LayerBucketAllReduce(model.layers, layers_per_bucket=2, small_bytes=1024, tail_layers=2)
    keys = [k[0] for k, _, _, _ in red.buckets if k[1] == torch.bfloat16]
    # layers 3 and 2 share a bucket; layers 1 and 0 (the last two of the backward) get one each
    assert sorted(map(str, keys)) == sorted(map(str, [0, ("tail", 1), ("tail", 0)]))
    for _, _, flat, params in red.buckets:
        assert sum(p.numel() for p in params) == flat.numel()
        assert all(p.grad.data_ptr() >= flat.data_ptr() for p in params)
    assert red.bytes == sum(p.numel() * p.element_size() for p in model.parameters())


def test_gemm_gradients_written_into_buckets_match_autograd():
    """The bucket-owned weights get dW written by their GEMM backward; the same model without a
    reducer gets plain autograd gradients: equal, and the reducer's accumulated tails are zeroed."""
    import copy

    from harness.block import loss_fn
    from harness.grad_sync import LayerBucketAllReduce, train_step
    cfg = tiny_cfg()
    model = make_model(cfg)
    plain = copy.deepcopy(model)
    reducer = LayerBucketAllReduce(model.layers, small_bytes=0)
    x = global_batch(cfg)
    for _ in range(2):                      # a second step must not accumulate onto the first
        train_step(model, x, reducer, 1, loss_fn)
    loss_fn(plain(x)).backward()
    for (n, a), (_, b) in zip(model.named_parameters(), plain.named_parameters()):
        torch.testing.assert_close(a.grad, b.grad, rtol=1e-5, atol=1e-7, msg=n)
    assert reducer.zero_tails and sum(t.numel() for t in reducer.zero_tails) < reducer.bytes // 4


def test_dead_rank_raises_instead_of_hanging():
    res = run_ranks(2, "die")
    assert res[1][0] == "error" and "planted" in res[1][1]
    assert res[0][0] == "error", res[0]      # its all-reduce ends with an error (peer gone / timeout)
