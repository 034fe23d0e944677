"""Data-parallel step on 2 GPUs (one process per GPU, NCCL over NVLink).

Each rank runs the device step on its half of a batch with the library's
bucketed gradient all-reduce attached; the reduced gradients must equal the
oracle's full-batch gradients (float64 adjudication),
be bit-identical on both ranks, and keep the replicas identical after AdamW.
Skipped when fewer than 2 GPUs are visible.
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CFG = dict(vocab_size=256, block_size=64, n_layer=2, n_head=4, n_embd=128)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from neuralsuite_b200 import GPTConfig, init_params

    cfg = GPTConfig(**CFG)
    r = np.random.default_rng(42)
    flat = init_params(cfg, r, ln_noise=0.05)
    idx = r.integers(0, cfg.vocab_size, (8, 64)).astype(np.int32)
    tgt = r.integers(0, cfg.vocab_size, (8, 64)).astype(np.int32)
    return cfg, flat, idx, tgt


def _rank(rank, world, port, out):
    from datetime import timedelta

    import torch.distributed as dist

    from neuralsuite_b200 import Comm, GPTModel

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    cfg, flat, idx, tgt = _inputs()
    per = idx.shape[0] // world
    m = GPTModel(cfg, max_batch=per)
    m.set_params(flat)
    comm = Comm(rank, world)
    m.set_comm(comm, world, bucket_floats=1 << 16)
    tok = torch.as_tensor(idx[rank * per:(rank + 1) * per], device="cuda")
    tg = torch.as_tensor(tgt[rank * per:(rank + 1) * per].reshape(-1), device="cuda")
    m.adamw_init(3e-4)
    m.forward(tok)
    m.loss_backward(tg)
    m.backward()
    torch.cuda.synchronize()
    np.save(os.path.join(out, f"grads{rank}.npy"), m.get_grads())
    loss = m.train_step(tok, tg)  # full step incl. AdamW, loss all-reduced
    np.save(os.path.join(out, f"params{rank}.npy"), m.get_params())
    np.save(os.path.join(out, f"loss{rank}.npy"), np.array([loss]))
    m.set_comm(None, 1)
    comm.destroy()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_data_parallel_matches_full_batch(port):
    from oracle import fp64
    from tests._util import close_report

    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank, args=(world, _free_port(), d), nprocs=world, start_method="spawn",
                           join=True)
        g0, g1 = np.load(os.path.join(d, "grads0.npy")), np.load(os.path.join(d, "grads1.npy"))
        p0, p1 = np.load(os.path.join(d, "params0.npy")), np.load(os.path.join(d, "params1.npy"))
        l0, l1 = float(np.load(os.path.join(d, "loss0.npy"))[0]), float(np.load(os.path.join(d, "loss1.npy"))[0])
    assert np.array_equal(g0.view(np.uint32), g1.view(np.uint32)), "ranks disagree after all-reduce"
    assert np.array_equal(p0.view(np.uint32), p1.view(np.uint32)), "replicas drifted after AdamW"
    assert l0 == l1
    cfg, flat, idx, tgt = _inputs()
    o = port.gpt(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd)
    o.set_params(flat)
    ref_loss, _ = o.fwd_bwd(idx.astype(np.float32), tgt.reshape(-1).astype(np.float32))
    ref = o.get_grads()
    _, _, g64 = fp64.gpt_fwd_bwd(flat, idx, tgt.reshape(-1), cfg.vocab_size, cfg.block_size,
                                 cfg.n_layer, cfg.n_head, cfg.n_embd)
    ok, info = close_report(g0, ref, g64)
    assert ok, info
    assert abs(l0 - ref_loss) < 1e-4 * abs(ref_loss)
