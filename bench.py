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
import os
import statistics
import subprocess
import sys
import tempfile
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
                    help="skip the reference CPU leg (it costs ~1-2 min: samples + one full step)")
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

def _reference_model():
    import oracle

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
    return g, r, cores, kind


def _reference_step(g, r, nseq):
    idx = r.integers(0, V, (nseq, T)).astype(np.float32)
    tgt = r.integers(0, V, nseq * T).astype(np.float32)
    t0 = time.perf_counter()
    g.fwd_bwd(idx, tgt)
    g.adamw_step()
    return nseq * T / (time.perf_counter() - t0)


def reference_run(steps, warmup, calibrate=True):
    """The NeuralSuite reference (oracle/_ref, built from its own sources) on
    the host cores.  Each step is a bounded sample of the workload: one of the
    8 sequences of a step (1024 tokens) through the full 12-layer model,
    forward + CrossEntropy + backward + AdamW.  With calibrate, one full
    8-sequence step (8192 tokens, the GPU arm's per-GPU batch) is timed once
    in the same run, so the per-token rate of the sample can be set against
    the rate of the real configuration (the reference's attention and its
    [B,H,T,T] probability cache scale with the batch).  Returns (median
    sample tokens/s, cores, kind, description, calibration dict or None)."""
    g, r, cores, kind = _reference_model()
    vals = []
    for i in range(warmup + steps):
        v = _reference_step(g, r, 1)
        if i >= warmup:
            vals.append(v)
    sample = statistics.median(vals)
    cal = None
    if calibrate:
        full = _reference_step(g, r, B_PER_GPU)
        cal = {"full_step_tokens_per_s": full, "full_step_tokens": B_PER_GPU * T,
               "sample_tokens_per_s": sample, "full_over_sample": full / sample,
               "note": "one full 8-sequence step timed once after the samples, same run"}
    desc = (f"1 of the 8 sequences of a step per timed step: {T} tokens through all {LAYERS} "
            f"layers (forward + CrossEntropy + backward + AdamW), {cores} host thread(s)")
    return sample, cores, kind, desc, cal


def run_reference(args, rank, world):
    if rank != 0:
        return
    value, cores, kind, desc, cal = reference_run(args.steps, args.warmup)
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": T / value * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (uniform byte tokens, seeded)",
        "config": {"workload": WORKLOAD,
                   "global_batch": "1 of the 8 sequences per timed step (bounded sample); "
                                   "one full 8-sequence step in calibration",
                   "seq_len": T, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind,
                         "sample": desc},
        "calibration": cal,
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
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix=f"ns_clocks_{self.index}_", suffix=".csv")
            self.f = os.fdopen(fd, "w")
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
        with open(self.path) as fh:
            lines = fh.readlines()
        os.unlink(self.path)
        for line in lines:
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


def gemm_roofline(torch, nk, presplit):
    """Times every GEMM shape of the step with CUDA events on the current
    stream (alone, warm, operands > L2 for the big ones) and returns step-
    weighted achieved TFLOP/s for all GEMMs and for the backward ones.
    presplit: the operands' tf32 lo parts are made once beforehand and passed
    in (ns_gemm_lo, the form the training step runs, where each producer
    writes the lo part of its output); otherwise ns_gemm splits them into its
    workspace inside every call."""
    dev = torch.device("cuda")
    tot_f = tot_t = bwd_f = bwd_t = 0.0
    launches = 0
    per = []
    for cnt, m, n, k, at, bt, bwd in gemm_shapes():
        A = torch.randn((k, m) if at else (m, k), device=dev)
        Bm = torch.randn((n, k) if bt else (k, n), device=dev)
        out = torch.empty(m, n, device=dev)
        kw = dict(a_trans=bool(at), b_trans=bool(bt), out=out)
        if presplit:
            kw.update(a_lo=nk.split_lo(A), b_lo=nk.split_lo(Bm))
        for _ in range(2):
            nk.gemm(A, Bm, **kw)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        torch.cuda.synchronize()
        s.record()
        for _ in range(reps):
            nk.gemm(A, Bm, **kw)
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
        del A, Bm, out, kw
    return tot_f / tot_t / 1e9, bwd_f / bwd_t / 1e9, tot_f / launches, tot_t / launches, per


def make_batches(rank, n_batches):
    """Seeded uniform byte tokens and targets of one rank (int32, host)."""
    r = np.random.default_rng(1000 + rank)
    tok = [r.integers(0, V, (B_PER_GPU, T)).astype(np.int32) for _ in range(n_batches)]
    tgt = [r.integers(0, V, (B_PER_GPU * T,)).astype(np.int32) for _ in range(n_batches)]
    return tok, tgt


def dp_checks(torch, dist, model, cfg, rank, world, n_batches):
    """Data-parallel correctness after the timed steps (untimed).

    replicas_identical: rank 0's parameter buffer broadcast to every rank and
    compared bit for bit with the rank's own.  Then one forward + loss +
    backward on every rank's first batch with the gradient all-reduce (no
    optimizer step), against rank 0 recomputing each rank's shard alone
    (world 1) on the same parameters: the global loss against the mean of the
    shard losses, and the all-reduced gradient against the mean of the shard
    gradients, |x - ref| <= 1e-5 + 1e-4 |ref|."""
    from neuralsuite_b200 import GPTModel

    mine = model.params()
    ref = mine.clone()
    dist.broadcast(ref, src=0)
    same = torch.tensor([1 if torch.equal(mine, ref) else 0], device="cuda", dtype=torch.int32)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    del ref
    tok, tgt = make_batches(rank, n_batches)
    model.forward(torch.from_numpy(tok[0]).cuda())
    model.loss_backward(torch.from_numpy(tgt[0]).cuda())
    model.backward()
    torch.cuda.synchronize()
    loss_dp = float(model.loss_tensor().item()) / world
    out = {"replicas_identical": bool(same.item() == 1)}
    if rank == 0:
        solo = GPTModel(cfg, max_batch=B_PER_GPU)
        solo.params().copy_(model.params())
        acc = torch.zeros(model.n_params, dtype=torch.float64, device="cuda")
        losses = []
        for r in range(world):
            t_r, g_r = make_batches(r, 1)
            solo.forward(torch.from_numpy(t_r[0]).cuda())
            losses.append(float(solo.loss_backward(torch.from_numpy(g_r[0]).cuda()).item()))
            solo.backward()
            acc += solo.grads().double()
        want = acc / world
        got = model.grads().double()
        err = (got - want).abs()
        bad = int((err > 1e-5 + 1e-4 * want.abs()).sum().item())
        loss_1 = sum(losses) / world
        out.update({
            "loss_dp": loss_dp, "loss_1gpu_recompute": loss_1,
            "loss_rel_err": abs(loss_dp - loss_1) / abs(loss_1),
            "grad_max_abs_err": float(err.max().item()), "grad_elements_outside_tol": bad,
            "ok": bool(out["replicas_identical"] and bad == 0
                       and abs(loss_dp - loss_1) <= 1e-5 + 1e-4 * abs(loss_1)),
        })
        del solo, acc, want, got, err
    dist.barrier()
    return out


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
    n_batches = 4  # distinct batches cycled through the timed steps
    tok_np, tgt_np = make_batches(rank, n_batches)
    host_tok = [torch.from_numpy(t).pin_memory() for t in tok_np]
    host_tgt = [torch.from_numpy(t).pin_memory() for t in tgt_np]
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

    dp = dp_checks(torch, dist, model, cfg, rank, world, n_batches) if world > 1 else None

    out = None
    if rank == 0:
        bf16_burst, bf16_sust, hbm, peak_src = peaks()
        all_tf, bwd_tf, flops_per_launch, ms_per_launch, per = gemm_roofline(torch, nk, True)
        all_tf_ws, bwd_tf_ws, _, _, per_ws = gemm_roofline(torch, nk, False)
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
                "avg_launch_ms": ms_per_launch,
                "operands": "tf32 lo parts made by the producers and passed in (ns_gemm_lo), "
                            "as the training step runs the products",
                "shapes": per,
                "split_in_call": {"achieved": all_tf_ws, "frac": all_tf_ws / peak_3x,
                                  "bwd_gemm_tflops": bwd_tf_ws,
                                  "note": "ns_gemm splitting both operands into its workspace "
                                          "inside every call", "shapes": per_ws},
            },
        }
        if dp is not None:
            out["dp_check"] = dp
            out["replicas_identical"] = dp["replicas_identical"]
    if world > 1:
        model.set_comm(None, 1)
        comm.destroy()
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            v, cores, kind, desc, cal = reference_run(steps=3, warmup=1)
            out["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": cores, "kind": kind,
                                   "sample": desc + "; median of 3 after 1 warm-up",
                                   "calibration": cal}
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
