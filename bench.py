"""Benchmark of the GPT training step on B200 (one process per GPU).

Workload (the 12-layer configuration the headline metric is quoted on):
GPTModel vocab 256, n_layer 12, n_embd 768, n_head 12, T = 1024, 8 sequences
per GPU of uniform random byte tokens, N(0, 0.02) weights (LayerNorm 1/0, bias
0), one forward + CrossEntropy + full backward (+ NCCL gradient all-reduce for
N > 1) + AdamW(lr 3e-4) step.  fp32 parameters, 3xTF32 GEMMs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  With N > 1 launch under torchrun; data
parallel with weak scaling (8 sequences per GPU).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "GPT train-step tokens/s at 1/2/4/8 B200; bwd GEMM TFLOP/s vs tensor peak"
V, BLOCK, LAYERS, HEADS, EMBD, T, B_PER_GPU = 256, 1024, 12, 12, 768, 1024, 8
LR = 3e-4
WORKLOAD = "GPTModel 12L/768/12h, T=1024, 8 seq/GPU, vocab 256, AdamW"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the reference CPU sample (it costs ~15-25 s)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops"), d.get("bf16_tflops_sustained"), d.get("hbm_gbs"), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


# ----------------------------------------------------------- reference CPU leg

def reference_sample(seconds_hint=False):
    """The NeuralSuite reference (oracle/_ref, built from its own sources) on
    the host cores: one sequence of 1024 tokens (one of the 8 sequences a GPU
    processes per step) through the full 12-layer model, forward +
    CrossEntropy + backward + AdamW.  Returns (tokens/s, cores, kind, sample
    description)."""
    import oracle

    Ts = T
    if oracle.ref_available():
        o = oracle.ref()
        cores = os.cpu_count() or 1
        o.set_threads(cores)
        kind = "reference"
    else:
        o = oracle.port()
        cores = 1
        kind = "port"
    g = o.gpt(V, BLOCK, LAYERS, HEADS, EMBD)
    r = np.random.default_rng(5)
    g.set_params((r.standard_normal(g.num_params()) * 0.02).astype(np.float32))
    g.adamw_init(LR)
    idx = r.integers(0, V, (1, Ts)).astype(np.float32)
    tgt = r.integers(0, V, Ts).astype(np.float32)
    t0 = time.perf_counter()
    g.fwd_bwd(idx, tgt)
    g.adamw_step()
    dt = time.perf_counter() - t0
    desc = (f"1 of the 8 sequences of a step: {Ts} tokens through all {LAYERS} layers "
            f"(forward + CrossEntropy + backward + AdamW), {cores} host thread(s)")
    return Ts / dt, cores, kind, desc


def run_reference(args, rank, world):
    if rank != 0:
        return
    vals = []
    for i in range(args.warmup + args.steps):
        v, cores, kind, desc = reference_sample()
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": T / value * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (uniform byte tokens, seeded)",
        "config": {"workload": WORKLOAD, "global_batch": "1 sequence sampled per step",
                   "seq_len": T, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind,
                         "sample": desc},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# ----------------------------------------------------------- clocks

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join(HERE, "gpurun_out", f"clocks_rank{index}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------- GEMM roofline

def gemm_shapes():
    """(count per step, M, N, K, a_trans, b_trans, is_backward) of every GEMM."""
    M, C, F = B_PER_GPU * T, EMBD, 4 * EMBD
    L = LAYERS
    return [
        (L, M, 3 * C, C, 0, 0, 0), (L, M, C, C, 0, 0, 0), (L, M, F, C, 0, 0, 0), (L, M, C, F, 0, 0, 0),
        (1, M, V, C, 0, 1, 0),
        (L, M, C, 3 * C, 0, 1, 1), (L, M, C, C, 0, 1, 1), (L, M, C, F, 0, 1, 1), (L, M, F, C, 0, 1, 1),
        (L, C, 3 * C, M, 1, 0, 1), (L, C, C, M, 1, 0, 1), (L, C, F, M, 1, 0, 1), (L, F, C, M, 1, 0, 1),
        (1, M, C, V, 0, 0, 1), (1, V, C, M, 1, 0, 1),
    ]


def gemm_roofline(torch, nk):
    """Times every GEMM shape of the step with CUDA events on the current
    stream (alone, warm, operands > L2 for the big ones) and returns step-
    weighted achieved TFLOP/s for all GEMMs and for the backward ones."""
    dev = torch.device("cuda")
    tot_f = tot_t = bwd_f = bwd_t = 0.0
    launches = 0
    per = []
    for cnt, m, n, k, at, bt, bwd in gemm_shapes():
        A = torch.randn((k, m) if at else (m, k), device=dev)
        Bm = torch.randn((n, k) if bt else (k, n), device=dev)
        out = torch.empty(m, n, device=dev)
        for _ in range(2):
            nk.gemm(A, Bm, a_trans=bool(at), b_trans=bool(bt), out=out)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        torch.cuda.synchronize()
        s.record()
        for _ in range(reps):
            nk.gemm(A, Bm, a_trans=bool(at), b_trans=bool(bt), out=out)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / reps
        flops = 2.0 * m * n * k
        per.append({"mnk": [m, n, k], "at": at, "bt": bt, "ms": round(ms, 4),
                    "tflops": round(flops / ms / 1e9, 1)})
        tot_f += cnt * flops
        tot_t += cnt * ms
        launches += cnt
        if bwd:
            bwd_f += cnt * flops
            bwd_t += cnt * ms
        del A, Bm, out
    return tot_f / tot_t / 1e9, bwd_f / bwd_t / 1e9, tot_f / launches, tot_t / launches, per


# ----------------------------------------------------------- our leg

def run_ours(args, rank, world, local):
    import torch

    torch.cuda.set_device(local)
    import torch.distributed as dist

    from neuralsuite_b200 import Comm, GPTConfig, GPTModel, init_params
    from neuralsuite_b200 import _lib
    from neuralsuite_b200 import kernels as nk

    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    lib = _lib.load()
    cfg = GPTConfig(V, BLOCK, LAYERS, HEADS, EMBD)
    model = GPTModel(cfg, max_batch=B_PER_GPU)
    flat = init_params(cfg, np.random.default_rng(1234))  # same weights on every rank
    model.set_params(flat)
    model.adamw_init(LR)
    comm = None
    if world > 1:
        comm = Comm(rank, world)
        model.set_comm(comm, world)
    r = np.random.default_rng(1000 + rank)
    n_batches = 4  # distinct batches cycled through the timed steps
    host_tok = [torch.from_numpy(r.integers(0, V, (B_PER_GPU, T)).astype(np.int32)).pin_memory()
                for _ in range(n_batches)]
    host_tgt = [torch.from_numpy(r.integers(0, V, (B_PER_GPU * T,)).astype(np.int32)).pin_memory()
                for _ in range(n_batches)]
    dev_tok = [t.cuda() for t in host_tok]
    dev_tgt = [t.cuda() for t in host_tgt]
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # -- device-resident leg: inputs already in HBM
    for i in range(args.warmup):
        model.train_step(dev_tok[i % n_batches], dev_tgt[i % n_batches], read_loss=False)
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    n0 = lib.ns_launch_count()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(args.steps):
        model.train_step(dev_tok[i % n_batches], dev_tgt[i % n_batches], read_loss=False)
    e.record()
    torch.cuda.synchronize()
    launches = lib.ns_launch_count() - n0
    barrier()
    ms = max_over_ranks(s.elapsed_time(e)) / args.steps
    clk = clocks.stop()
    loss_dev = float(model.loss_tensor().item()) / world  # device holds the sum over ranks

    # -- end-to-end leg through the public API: pinned host tokens/targets in,
    # loss out, every step
    barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tok_buf, tgt_buf = torch.empty_like(dev_tok[0]), torch.empty_like(dev_tgt[0])
    s2.record()
    last_loss = None
    for i in range(args.steps):
        tok_buf.copy_(host_tok[i % n_batches], non_blocking=True)
        tgt_buf.copy_(host_tgt[i % n_batches], non_blocking=True)
        last_loss = model.train_step(tok_buf, tgt_buf, read_loss=True)
    e2.record()
    torch.cuda.synchronize()
    barrier()
    ms_e2e = max_over_ranks(s2.elapsed_time(e2)) / args.steps
    h2d = host_tok[0].numel() * 4 + host_tgt[0].numel() * 4
    d2h = 4 * 4

    tokens_per_step = world * B_PER_GPU * T
    value = tokens_per_step / (ms / 1e3)
    e2e_value = tokens_per_step / (ms_e2e / 1e3)

    out = None
    if rank == 0:
        bf16_burst, bf16_sust, hbm, peak_src = peaks()
        all_tf, bwd_tf, flops_per_launch, ms_per_launch, per = gemm_roofline(torch, nk)
        nk.kernel_health()
        tf32_peak = bf16_burst / 2.0  # dense TF32 = half the dense BF16 rate (datasheet ratio)
        peak_3x = tf32_peak / 3.0     # 3xTF32: three tensor passes per fp32 product
        traffic = None
        tp = os.path.join(HERE, "profiles", "gemm_traffic.json")
        if os.path.exists(tp):
            traffic = json.load(open(tp)).get("dram_bytes_per_launch")
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: uniform random byte tokens, seeded N(0,0.02) weights",
            "config": {"workload": WORKLOAD, "model": "GPTModel 12L/768/12h vocab 256",
                       "global_batch": world * B_PER_GPU, "seq_len": T,
                       "parallelism": f"dp{world}",
                       "l2": "working set (344 MB params + >4 GB activations) exceeds the 126 MB L2; no flush"},
            "tokens_per_step": tokens_per_step,
            "loss_last_step": loss_dev, "loss_e2e_last": last_loss,
            "gpu_launches": int(launches),
            "clocks": clk,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "ms_per_step": ms_e2e,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": {
                "bound": "tensor", "kernel": "ns_gemm (tcgen05 3xTF32), all GEMM shapes of the step",
                "achieved": all_tf, "peak": peak_3x, "unit": "TFLOP/s", "frac": all_tf / peak_3x,
                "traffic": traffic,
                "peak_source": f"{peak_src}: bf16 burst {bf16_burst} TF/s / 2 (TF32) / 3 (3xTF32 passes)",
                "achieved_is": "algorithmic fp32 FLOP (2MNK) per launch / CUDA-event launch time",
                "bwd_gemm_tflops": bwd_tf, "bwd_gemm_frac": bwd_tf / peak_3x,
                "bwd_tensor_issue_frac_of_tf32_peak": 3 * bwd_tf / tf32_peak,
                "algorithmic_flops_per_launch": flops_per_launch,
                "avg_launch_ms": ms_per_launch, "shapes": per,
            },
        }
    if world > 1:
        model.set_comm(None, 1)
        comm.destroy()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            v, cores, kind, desc = reference_sample()
            out["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": kind,
                                   "sample": desc}
        print(json.dumps(out), flush=True)


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
