"""Host-side checks of the data-parallel step (no GPU): the gradient bucket plan
and the arithmetic the GPU path relies on, run as world_size-2 gloo ranks.

The GPU step divides the cross-entropy gradient by rows * world_size and sums
the per-rank gradients with NCCL.  Here two CPU ranks each run the oracle (the
reference-exact C restatement) on their half of a batch, sum their gradients
with a gloo all-reduce, divide by world_size, and must recover the oracle's
full-batch gradient.
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch.multiprocessing as mp

from neuralsuite_b200.model import GPTConfig, init_params, param_shapes, plan_buckets


def test_bucket_plan_covers_every_gradient_once_in_backward_order():
    cfg = GPTConfig(256, 1024, 12, 12, 768)
    total = sum(int(np.prod(s)) for s in param_shapes(cfg))
    for cap in (0, 1 << 22, 1000):
        b = plan_buckets(cfg, cap)
        covered = np.zeros(total, np.int8)
        for lo, hi in b:
            assert 0 <= lo < hi <= total
            if cap:
                assert hi - lo <= cap
            covered[lo:hi] += 1
        assert covered.min() == 1 and covered.max() == 1
        # launch order follows the backward: the bucket that ends with ln_f (the
        # end of the flat buffer) goes before the one that starts with wte.
        last = next(i for i, (lo, hi) in enumerate(b) if hi == total)
        first = next(i for i, (lo, hi) in enumerate(b) if lo == 0)
        assert last < first
    assert len(plan_buckets(cfg, 0)) == cfg.n_layer + 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_rank(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    import oracle

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    cfg = GPTConfig(64, 16, 2, 2, 32)
    r = np.random.default_rng(0)
    flat = init_params(cfg, r, ln_noise=0.05)
    idx = r.integers(0, cfg.vocab_size, (4, 16)).astype(np.float32)
    tgt = r.integers(0, cfg.vocab_size, 64).astype(np.float32)
    shard = slice(rank * 2, rank * 2 + 2)
    g = oracle.port().gpt(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd)
    g.set_params(flat)
    loss, _ = g.fwd_bwd(idx[shard], tgt.reshape(4, 16)[shard].reshape(-1))
    grads = torch.from_numpy(g.get_grads() / world)
    lt = torch.tensor([loss / world])
    dist.all_reduce(grads)
    dist.all_reduce(lt)
    if rank == 0:
        np.save(os.path.join(out_dir, "dp_grads.npy"), grads.numpy())
        np.save(os.path.join(out_dir, "dp_loss.npy"), lt.numpy())
    dist.destroy_process_group()


def test_two_rank_gradient_sum_equals_full_batch(port):
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_dp_rank, args=(world, _free_port(), d), nprocs=world,
                           start_method="spawn", join=True)
        grads = np.load(os.path.join(d, "dp_grads.npy"))
        loss = float(np.load(os.path.join(d, "dp_loss.npy"))[0])
    cfg = GPTConfig(64, 16, 2, 2, 32)
    r = np.random.default_rng(0)
    flat = init_params(cfg, r, ln_noise=0.05)
    idx = r.integers(0, cfg.vocab_size, (4, 16)).astype(np.float32)
    tgt = r.integers(0, cfg.vocab_size, 64).astype(np.float32)
    g = port.gpt(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd)
    g.set_params(flat)
    full_loss, _ = g.fwd_bwd(idx, tgt)
    assert abs(loss - full_loss) < 1e-5
    ref = g.get_grads()
    assert np.allclose(grads, ref, rtol=1e-4, atol=1e-6), np.abs(grads - ref).max()


def _failing_rank(rank, world, port):
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        raise RuntimeError("injected failure on rank 1 before the gradient all-reduce")
    t = torch.ones(4)
    dist.all_reduce(t)  # rank 1 never joins: must end with an error, not hang


def test_rank_failure_surfaces_as_an_error():
    """A rank that dies before the exchange: the job ends with an error within
    the process-group timeout instead of waiting forever (host-side failure
    injection; no GPU involved)."""
    with pytest.raises(Exception):
        mp.start_processes(_failing_rank, args=(2, _free_port()), nprocs=2, start_method="spawn",
                           join=True)
