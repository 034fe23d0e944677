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
    ap.add_argument("--case", default="step",
                    choices=["step", "c1", "c2", "c3", "c5", "decode", "lstm", "gemm", "attn",
                             "bw", "conv"],
                    help="step: the training-step benchmark (default, the one-line contract); "
                         "c1 / c2 / c3: the 4-layer/128 step, the MatMul sweep, the "
                         "MultiHeadAttention layer at B8/T1024/H12, each beside the reference "
                         "on the host cores; c5: the diffusion U-Net step (data parallel under "
                         "torchrun); decode: KV-cache decoding of the 12-layer model; "
                         "gemm / attn / bw / conv: single-kernel cases for profilers")
    ap.add_argument("--shape", default="",
                    help="gemm: M,N,K[,a_trans,b_trans]; attn: B,T,H,D; bw: M,C,V; "
                         "conv: B,IC,H,W,OC,k,stride,pad")
    ap.add_argument("--reps", type=int, default=3, help="launches per kernel case")
    ap.add_argument("--engine", type=int, default=0, help="gemm / attn engine of the case")
    ap.add_argument("--epilogue", type=int, default=0, help="gemm case epilogue")
    ap.add_argument("--presplit", action="store_true", help="gemm case: pass the lo parts in")
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
            t_r, g_r = make_batches(r, n_batches)  # the same draws as rank r's own
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

    # -- where the data-parallel step loses time to communication (untimed
    # extra steps, each read back): the compute stream's wait for the
    # gradient all-reduces after its backward, and their span
    comm_info = None
    if world > 1:
        model.set_comm_timing(True)
        exposed, span = [], []
        for i in range(5):
            model.train_step(dev_tok[i % n_batches], dev_tgt[i % n_batches], read_loss=False)
            x, y = model.comm_times()
            exposed.append(x)
            span.append(y)
        model.set_comm_timing(False)

        # forward + loss + backward (no optimizer step, so the replicas stay
        # identical), with the all-reduce and then with the communicator detached
        def fwd_bwd_ms():
            barrier()
            torch.cuda.synchronize()
            s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s3.record()
            for i in range(5):
                model.forward(dev_tok[i % n_batches])
                model.loss_backward(dev_tgt[i % n_batches])
                model.backward()
            e3.record()
            torch.cuda.synchronize()
            return max_over_ranks(s3.elapsed_time(e3) / 5)

        fb_dp = fwd_bwd_ms()
        model.set_comm(None, 1)
        fb_local = fwd_bwd_ms()
        model.set_comm(comm, world)
        comm_info = {"exposed_ms": max_over_ranks(statistics.median(exposed)),
                     "allreduce_span_ms": max_over_ranks(statistics.median(span)),
                     "fwd_bwd_ms_allreduce": fb_dp, "fwd_bwd_ms_local": fb_local,
                     "how": "median of 5 extra steps, max over ranks; exposed = the compute "
                            "stream's wait for the all-reduces after its own backward; "
                            "fwd_bwd_ms_* = forward + loss + backward (no optimizer step), mean "
                            "of 5, max over ranks, with the all-reduce and with the "
                            "communicator detached"}

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
        if comm_info is not None:
            out["comm"] = comm_info
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


# ----------------------------------------------------------- other configurations

def _event_ms(torch, fn, reps, warm=1):
    """Median CUDA-event time (ms) of fn over reps launches on the current stream."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return statistics.median(out)


def _host_ms(fn, reps, warm=1):
    """Median wall time (ms) of a host call (the reference's MedianMs pattern,
    benchmarks/benchmark.cpp:37-50)."""
    for _ in range(warm):
        fn()
    out = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        out.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(out)


def _ref_or_none(args):
    import oracle

    if args.no_cpu_baseline or not oracle.ref_available():
        return None
    o = oracle.ref()
    o.set_threads(os.cpu_count() or 1)
    return o


def case_c1(args, torch):
    """GPTModel 4 layers / n_embd 128 / 4 heads, T=64, B=8, vocab 256, AdamW
    lr 3e-4: the full training step (forward + CrossEntropy + backward +
    AdamW) from plain stream launches and from a CUDA-graph replay of the
    same launches; the forward + CrossEntropy + backward part alone (the
    reference's benchmark --train pattern, benchmarks/benchmark.cpp:118-157);
    the reference's full step on the host cores beside it."""
    from neuralsuite_b200 import GPTConfig, GPTModel, init_params

    Vc, L, H, C, Tc, Bc = 256, 4, 4, 128, 64, 8
    cfg = GPTConfig(Vc, Tc, L, H, C)
    flat = init_params(cfg, np.random.default_rng(1234))
    m = GPTModel(cfg, max_batch=Bc)
    m.set_params(flat)
    m.adamw_init(3e-4)
    r = np.random.default_rng(7)
    tok = torch.as_tensor(r.integers(0, Vc, (Bc, Tc)).astype(np.int32), device="cuda")
    tgt = torch.as_tensor(r.integers(0, Vc, Bc * Tc).astype(np.int32), device="cuda")
    steps = max(args.steps, 20)

    def step():
        m.train_step(tok, tgt, read_loss=False)

    def fwd_bwd():
        m.forward(tok)
        m.loss_backward(tgt)
        m.backward()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ms_step = _event_ms(torch, lambda: [step() for _ in range(steps)], 3) / steps
    ms_fb = _event_ms(torch, lambda: [fwd_bwd() for _ in range(steps)], 3) / steps
    graph_ms, graph_note = None, None
    try:
        g = torch.cuda.CUDAGraph()
        sidestream = torch.cuda.Stream()
        sidestream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(sidestream):
            step()
        torch.cuda.current_stream().wait_stream(sidestream)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            step()
        graph_ms = _event_ms(torch, lambda: [g.replay() for _ in range(steps)], 3) / steps
        del g
    except Exception as ex:  # capture is reported, not required
        graph_note = f"capture failed: {ex}"
    toks = Bc * Tc
    out = {"case": "c1", "workload": "GPTModel 4L/128/4h, T=64, B=8, vocab 256, AdamW lr 3e-4",
           "unit": "tokens/s", "tokens_per_step": toks,
           "step_us": ms_step * 1e3, "step_tokens_per_s": toks / ms_step * 1e3,
           "fwd_bwd_us": ms_fb * 1e3, "fwd_bwd_tokens_per_s": toks / ms_fb * 1e3,
           "graph_step_us": None if graph_ms is None else graph_ms * 1e3,
           "graph_step_tokens_per_s": None if graph_ms is None else toks / graph_ms * 1e3,
           "graph_note": graph_note,
           "roofline": "latency-bound (2.62 GFLOP per 512-token step); no roofline fraction"}
    o = _ref_or_none(args)
    if o is not None:
        gr = o.gpt(Vc, Tc, L, H, C)
        gr.set_params(flat)
        gr.adamw_init(3e-4)
        idx, tg = tok.cpu().numpy().astype(np.float32), tgt.cpu().numpy().astype(np.float32)

        def ref_step():
            gr.fwd_bwd(idx, tg)
            gr.adamw_step()

        rms = _host_ms(ref_step, 10)
        rfb = _host_ms(lambda: gr.fwd_bwd(idx, tg), 10)
        out["reference"] = {"step_ms": rms, "step_tokens_per_s": toks / rms * 1e3,
                            "fwd_bwd_ms": rfb, "fwd_bwd_tokens_per_s": toks / rfb * 1e3,
                            "cores": os.cpu_count(), "how": "median of 10 after 1 warm-up"}
    return out


def case_c2(args, torch):
    """The MatMul sweep: X[M,K], W[K,N], dY[M,N] ~ N(0,1); Y = X.W, dX = dY.W^T,
    dW = X^T.dY per shape, each a single ns_gemm call on fresh operands (the
    3xTF32 operand split inside the call), beside the reference's MatMul
    (src/tensor.cpp:198-271) on the host cores (its Transpose copies are made
    outside the timed region)."""
    from neuralsuite_b200 import kernels as nk

    bf16_burst, _, _, src = peaks()
    peak3 = bf16_burst / 2 / 3
    o = _ref_or_none(args)
    rows = []
    for M, K, N in [(512, 128, 512), (8192, 768, 3072), (8192, 3072, 768), (16384, 1024, 4096)]:
        g = torch.Generator(device="cuda").manual_seed(M + K + N)
        X = torch.randn(M, K, device="cuda", generator=g)
        W = torch.randn(K, N, device="cuda", generator=g)
        dY = torch.randn(M, N, device="cuda", generator=g)
        fl = 2.0 * M * N * K
        row = {"mkn": [M, K, N], "gflop": fl / 1e9}
        forms = {"Y": (X, W, False, False), "dX": (dY, W, False, True), "dW": (X, dY, True, False)}
        for name, (A, Bm, at, bt) in forms.items():
            ms = _event_ms(torch, lambda: nk.gemm(A, Bm, a_trans=at, b_trans=bt), max(args.reps, 5))
            row[name] = {"ms": ms, "tflops": fl / ms / 1e9, "frac": fl / ms / 1e9 / peak3}
        if o is not None:
            Xh, Wh, dYh = X.cpu().numpy(), W.cpu().numpy(), dY.cpu().numpy()
            host = {"Y": (Xh, Wh), "dX": (dYh, np.ascontiguousarray(Wh.T)),
                    "dW": (np.ascontiguousarray(Xh.T), dYh)}
            for name, (A, Bm) in host.items():
                ms = _host_ms(lambda: o.matmul(A, Bm), 3)
                row[name]["reference_ms"] = ms
                row[name]["reference_gflops"] = fl / ms / 1e6
        rows.append(row)
        del X, W, dY
    return {"case": "c2", "workload": "MatMul sweep, fp32 N(0,1) operands", "unit": "TFLOP/s",
            "peak": peak3, "peak_source": f"{src}: bf16 burst {bf16_burst} / 2 (TF32) / 3 (3xTF32)",
            "reference_cores": os.cpu_count() if o is not None else None, "shapes": rows}


def case_c3(args, torch):
    """MultiHeadAttention layer, B=8, T=1024, 12 heads, n_embd 768: forward
    (c_attn + causal attention + c_proj) and backward (the four projection
    gradients, dqkv, dx) composed from the C ABI, and the attention core
    alone, beside the reference layer's Forward + Backward on the host."""
    from neuralsuite_b200 import _lib
    from neuralsuite_b200 import kernels as nk

    Bc, Tc, H, C = 8, 1024, 12, 768
    D = C // H
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(Bc * Tc, C, device="cuda", generator=g)
    dy = torch.randn(Bc * Tc, C, device="cuda", generator=g)
    wa = torch.randn(C, 3 * C, device="cuda", generator=g) * 0.02
    ba = torch.zeros(3 * C, device="cuda")
    wp = torch.randn(C, C, device="cuda", generator=g) * 0.02
    bp = torch.zeros(C, device="cuda")
    st = {}

    def fwd():
        st["qkv"] = nk.gemm(x, wa, epilogue=_lib.EPI_BIAS, bias=ba)
        st["att"], st["lse"] = nk.attn_fwd(st["qkv"], Bc, Tc, H, D)
        st["y"] = nk.gemm(st["att"], wp, epilogue=_lib.EPI_BIAS, bias=bp)

    def bwd():
        nk.gemm(st["att"], dy, a_trans=True)
        nk.bias_grad(dy)
        datt = nk.gemm(dy, wp, b_trans=True)
        dqkv = nk.attn_bwd(st["qkv"], st["att"], datt, st["lse"], Bc, Tc, H, D)
        nk.gemm(x, dqkv, a_trans=True)
        nk.bias_grad(dqkv)
        nk.gemm(dqkv, wa, b_trans=True)

    reps = max(args.reps, 5)
    f_ms = _event_ms(torch, fwd, reps)
    fwd()
    b_ms = _event_ms(torch, bwd, reps)
    datt = nk.gemm(dy, wp, b_trans=True)
    cf = _event_ms(torch, lambda: nk.attn_fwd(st["qkv"], Bc, Tc, H, D), reps)
    cb = _event_ms(torch, lambda: nk.attn_bwd(st["qkv"], st["att"], datt, st["lse"], Bc, Tc, H, D),
                   reps)
    bf16_burst, _, _, src = peaks()
    peak3 = bf16_burst / 2 / 3
    core_f, core_b = 4.0 * Bc * H * D * Tc * (Tc + 1) / 2, 8.0 * Bc * H * D * Tc * (Tc + 1) / 2
    proj_f = 2.0 * Bc * Tc * C * 4 * C
    out = {"case": "c3", "workload": "MultiHeadAttention B=8, T=1024, H=12, C=768 (D=64)",
           "layer_fwd_ms": f_ms, "layer_bwd_ms": b_ms,
           "layer_fwd_tflops": (core_f + proj_f) / f_ms / 1e9,
           "layer_bwd_tflops": (core_b + 2 * proj_f) / b_ms / 1e9,
           "core_fwd_ms": cf, "core_bwd_ms": cb,
           "core_fwd_tflops": core_f / cf / 1e9, "core_bwd_tflops": core_b / cb / 1e9,
           "core_fwd_frac": core_f / cf / 1e9 / peak3, "core_bwd_frac": core_b / cb / 1e9 / peak3,
           "peak": peak3, "peak_source": f"{src}: bf16 burst {bf16_burst} / 2 / 3",
           "flops_note": "causal triangle: core fwd 4*B*H*D*T(T+1)/2 (S, O), bwd "
                         "8*B*H*D*T(T+1)/2 (dP, dV, dQ, dK; the recomputed S not counted); "
                         "projections 2*M*C*4C forward, twice that backward"}
    o = _ref_or_none(args)
    if o is not None:
        xh = x.cpu().numpy().reshape(Bc, Tc, C)
        dyh = dy.cpu().numpy().reshape(Bc, Tc, C)
        wah, bah, wph, bph = (t.cpu().numpy() for t in (wa, ba, wp, bp))
        rms = _host_ms(lambda: o.mha(Bc, Tc, C, H, wah, bah, wph, bph, xh, dyh), 1)
        out["reference"] = {"layer_fwd_bwd_ms": rms, "cores": os.cpu_count(),
                            "how": "one Forward + Backward after 1 warm-up"}
    return out


def unet_flops(B, in_ch=3, base=64, S=64):
    """Algorithmic FLOP of one U-Net training step: 3 x 2*MNK per convolution
    (forward, weight gradient, input gradient; conv_in has no input
    gradient), M = output channels, N = output pixels * B, K = 9 * input
    channels."""
    convs = [(in_ch, base, S), (base, 2 * base, S // 2), (2 * base, 4 * base, S // 4),
             (4 * base, 2 * base, S // 2), (2 * base, base, S), (base, in_ch, S)]
    convs += [(c, c, s) for c, s in ((base, S), (2 * base, S // 2), (4 * base, S // 4),
                                      (2 * base, S // 2), (base, S))]
    total = 0.0
    for i, (ic, oc, s) in enumerate(convs):
        f = 2.0 * oc * (B * s * s) * 9 * ic
        total += f * (2 if i == 0 else 3)
    return total


def case_c5(args, torch):
    """The diffusion U-Net training step of config 5: 64x64x3 images N(0,1),
    base channels 64, noise target N(0,1), MSELoss, AdamW, 32 images per GPU;
    data parallel (gradient all-reduce over NCCL) when launched under
    torchrun.  images/s over all ranks (max-over-ranks step time), the
    convolutions' algorithmic TFLOP/s, the reference's step on the host."""
    import torch.distributed as dist

    from neuralsuite_b200 import Comm, UNet

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    B = 32
    net = UNet(3, 64, 64, max_batch=B)
    r = np.random.default_rng(77)
    net.set_params((r.standard_normal(net.n_params) * 0.02).astype(np.float32))
    net.adamw_init(1e-4)
    comm = None
    if world > 1:
        comm = Comm(rank, world)
        net.set_comm(comm, world)
    rr = np.random.default_rng(100 + rank)
    xs = [torch.as_tensor(rr.standard_normal((B, 3, 64, 64)).astype(np.float32), device="cuda")
          for _ in range(2)]
    ts = [torch.as_tensor(rr.standard_normal((B, 3, 64, 64)).astype(np.float32), device="cuda")
          for _ in range(2)]
    for i in range(max(args.warmup, 3)):
        net.train_step(xs[i % 2], ts[i % 2], read_loss=False)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    steps = max(args.steps, 10)
    s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for i in range(steps):
        net.train_step(xs[i % 2], ts[i % 2], read_loss=False)
    e0.record()
    torch.cuda.synchronize()
    ms = s0.elapsed_time(e0) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        net.set_comm(None, 1)
        comm.destroy()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return None
    bf16_burst, _, _, src = peaks()
    fl = unet_flops(B)
    out = {"case": "c5", "workload": "diffusion U-Net, 64x64x3, base 64, 32 images/GPU, MSE, AdamW",
           "n_gpus": world, "step_ms": ms, "images_per_s": world * B / ms * 1e3,
           "conv_tflops_per_gpu": fl / ms / 1e9, "frac_of_3xtf32_peak": fl / ms / 1e9 / (bf16_burst / 6),
           "peak_source": src}
    o = _ref_or_none(args) if world == 1 else None
    if o is not None:
        from oracle import RefUNet

        ref_net = RefUNet(o, 3, 64, 64)
        ref_net.set_params((r.standard_normal(ref_net.n) * 0.02).astype(np.float32))
        ref_net.adamw_init(1e-4)
        xb = xs[0][:2].cpu().numpy()
        tb = ts[0][:2].cpu().numpy()

        def ref_step():
            ref_net.fwd_bwd(xb, tb)
            ref_net.adamw_step()

        rms = _host_ms(ref_step, 2)
        out["reference"] = {"images_per_s": 2 / rms * 1e3, "step_ms_for_2_images": rms,
                            "cores": os.cpu_count(), "sample": "2 of the 32 images per step"}
    return out


def case_lstm(args, torch):
    """BiLSTM forward + backward at a CRNN size (T 64 positions, 32 images,
    256 features, 256 hidden per direction), beside the reference's BiLSTM
    on the host cores; FLOP = 3 products x 2 directions x (input projection +
    recurrence) of 2*T*B*4H*(IN + H) each."""
    from neuralsuite_b200 import kernels as nk

    T, B, IN, H = 64, 32, 256, 256
    r = np.random.default_rng(8)
    n1 = 4 * H * IN + 4 * H * H + 8 * H
    p = torch.as_tensor((r.standard_normal(2 * n1) / 16).astype(np.float32), device="cuda")
    x = torch.as_tensor(r.standard_normal((T, B, IN)).astype(np.float32), device="cuda")
    d = torch.as_tensor(r.standard_normal((T, B, 2 * H)).astype(np.float32), device="cuda")
    ms = _event_ms(torch, lambda: nk.lstm_fwd_bwd(x, p, d, H, True), max(args.reps, 5))
    fl = 3 * 2 * 2.0 * T * B * 4 * H * (IN + H)
    out = {"case": "lstm", "workload": "BiLSTM T=64, B=32, IN=256, H=256, forward + backward",
           "ms": ms, "tflops": fl / ms / 1e9,
           "note": "the recurrence is 2 x 64 sequential steps each way, one cooperative kernel "
                   "per direction and pass (a grid barrier between steps)"}
    o = _ref_or_none(args)
    if o is not None:
        ph, xh, dh = p.cpu().numpy(), x.cpu().numpy(), d.cpu().numpy()
        rms = _host_ms(lambda: o.lstm(xh, ph, dh, H, True), 2)
        out["reference"] = {"ms": rms, "cores": os.cpu_count()}
    return out


def case_decode(args, torch):
    """KV-cache decoding (GPTModel::ForwardWithKVCache) of the 12-layer/768
    model: a prompt by prefill, then timed decode steps (CUDA events over
    consecutive steps), for 1 and 8 sequences at a short and a long context.
    Roofline: a step must read every weight once (86,039,040 floats) and the
    cached K and V of every sequence and layer; achieved GB/s = those bytes /
    step time, against the measured HBM copy bandwidth.  The reference's
    ForwardWithKVCache is timed on the host at the short context."""
    from neuralsuite_b200 import Decoder, GPTConfig, GPTModel, init_params

    cfg = GPTConfig(V, BLOCK, LAYERS, HEADS, EMBD)
    flat = init_params(cfg, np.random.default_rng(1234))
    _, _, hbm, src = peaks()
    steps = max(args.steps, 16)
    rows = []
    m = GPTModel(cfg, max_batch=8)
    m.set_params(flat)
    for B in (1, 8):
        dec = Decoder(m, max_batch=B)
        for ctx in (64, 960):
            dec.clear()
            r = np.random.default_rng(ctx + B)
            dec.prefill(r.integers(0, V, (B, ctx)))
            toks = [torch.as_tensor(r.integers(0, V, B).astype(np.int32), device="cuda")
                    for _ in range(steps + 2)]
            for i in range(2):
                dec.step(toks[i], ctx + i)
            torch.cuda.synchronize()
            s0, e0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record()
            for i in range(steps):
                dec.step(toks[2 + i], ctx + 2 + i)
            e0.record()
            torch.cuda.synchronize()
            ms = s0.elapsed_time(e0) / steps
            n_mid = ctx + 2 + steps // 2  # cached positions at the middle step
            nbytes = 4 * (m.n_params + B * LAYERS * 2 * EMBD * n_mid)
            rows.append({"sequences": B, "context": n_mid, "step_ms": ms,
                         "tokens_per_s": B / ms * 1e3, "bytes_per_step": nbytes,
                         "achieved_gbs": nbytes / ms / 1e6, "frac": nbytes / ms / 1e6 / hbm})
        del dec
    out = {"case": "decode", "workload": "GPTModel 12L/768/12h KV-cache decoding",
           "peak_gbs": hbm, "peak_source": src, "rows": rows}
    o = _ref_or_none(args)
    if o is not None:
        g = o.gpt(V, BLOCK, LAYERS, HEADS, EMBD)
        g.set_params(flat)
        g.clear_kv()
        r = np.random.default_rng(9)
        prompt = r.integers(0, V, 64)
        for p, t in enumerate(prompt):
            g.decode(int(t), p)
        ts = []
        for i in range(4):
            t0 = time.perf_counter()
            g.decode(int(r.integers(0, V)), 64 + i)
            ts.append(time.perf_counter() - t0)
        out["reference"] = {"sequences": 1, "context": 66, "step_ms": statistics.median(ts) * 1e3,
                            "tokens_per_s": 1.0 / statistics.median(ts), "cores": os.cpu_count()}
    return out


def case_kernel(args, torch):
    """Single-kernel cases sized for profiler captures (a few GB at most)."""
    from neuralsuite_b200 import kernels as nk

    dev = torch.device("cuda")
    torch.manual_seed(0)
    shape = [int(v) for v in args.shape.split(",")] if args.shape else []
    if args.case == "gemm":
        M, N, K = shape[:3]
        at, bt = (bool(shape[3]), bool(shape[4])) if len(shape) > 4 else (False, False)
        nk.set_gemm_engine(args.engine)
        A = torch.randn((K, M) if at else (M, K), device=dev)
        Bm = torch.randn((N, K) if bt else (K, N), device=dev)
        kw = {"out": torch.empty(M, N, device=dev), "epilogue": args.epilogue}
        if args.epilogue in (1, 2, 3):
            kw["bias"] = torch.randn(N, device=dev)
        if args.epilogue in (3, 4):
            kw["aux"] = torch.randn(M, N, device=dev)
        if args.presplit:
            kw.update(a_lo=nk.split_lo(A), b_lo=nk.split_lo(Bm))
        ms = _event_ms(torch, lambda: nk.gemm(A, Bm, a_trans=at, b_trans=bt, **kw), args.reps, 0)
        nk.set_gemm_engine(0)
        out = {"case": "gemm", "mnk": [M, N, K], "a_trans": at, "b_trans": bt,
               "epilogue": args.epilogue, "presplit": args.presplit, "ms": ms,
               "tflops": 2.0 * M * N * K / ms / 1e9}
    elif args.case == "conv":
        Bc, IC, H, W, OC, kk, st, pd = shape[:8] if shape else (32, 64, 64, 64, 3, 3, 1, 1)
        OH, OW = (H + 2 * pd - kk) // st + 1, (W + 2 * pd - kk) // st + 1
        x = torch.randn(Bc, IC, H, W, device=dev)
        w = torch.randn(OC, IC, kk, kk, device=dev) * 0.05
        bias = torch.randn(OC, device=dev)
        dy = torch.randn(Bc, OC, OH, OW, device=dev)
        f = _event_ms(torch, lambda: nk.conv2d_fwd(x, w, bias, stride=st, pad=pd), args.reps, 0)
        b = _event_ms(torch, lambda: nk.conv2d_bwd(x, dy, w, stride=st, pad=pd), args.reps, 0)
        fl = 2.0 * OC * Bc * OH * OW * IC * kk * kk
        out = {"case": "conv", "shape": [Bc, IC, H, W, OC, kk, st, pd], "fwd_ms": f, "bwd_ms": b,
               "fwd_tflops": fl / f / 1e9, "bwd_tflops": 2 * fl / b / 1e9}
    elif args.case == "attn":
        Bc, Tc, H, D = shape[:4]
        qkv = torch.randn(Bc * Tc, 3 * H * D, device=dev)
        dout = torch.randn(Bc * Tc, H * D, device=dev)
        nk.attn_set_engine(args.engine)
        o, lse = nk.attn_fwd(qkv, Bc, Tc, H, D)
        f = _event_ms(torch, lambda: nk.attn_fwd(qkv, Bc, Tc, H, D), args.reps, 0)
        b = _event_ms(torch, lambda: nk.attn_bwd(qkv, o, dout, lse, Bc, Tc, H, D), args.reps, 0)
        nk.attn_set_engine(0)
        out = {"case": "attn", "bthd": [Bc, Tc, H, D], "engine": args.engine, "fwd_ms": f,
               "bwd_ms": b}
    else:
        M, C, Vc = shape[:3] if shape else (8192, 768, 256)
        F = 4 * C
        rn = lambda *sh: torch.randn(*sh, device=dev)
        x, resid, raw = rn(M, C), rn(M, C), rn(M, C)
        g, b, bias = rn(C), rn(C), rn(C)
        dy3, pre3, dyq, logits = rn(M, F), rn(M, F), rn(M, 3 * C), rn(M, Vc)
        tgt = torch.randint(0, Vc, (M,), device=dev, dtype=torch.int32)
        tok = torch.randint(0, Vc, (M // 1024, 1024), device=dev, dtype=torch.int32)
        wte, wpe = rn(Vc, C), rn(1024, C)
        P = 86_039_040
        params, grads = rn(P), rn(P)
        mm, vv = torch.zeros(P, device=dev), torch.zeros(P, device=dev)
        _, _, _, mean, rstd = nk.layernorm_fwd_ex(x, g, b)
        cases = [
            ("ln_fwd_ex (resid + LayerNorm + lo)", (5 * M * C + 2 * M) * 4,
             lambda: nk.layernorm_fwd_ex(raw, g, b, bias=bias, resid=resid)),
            ("ln_bwd (+ dresid)", 4 * M * C * 4, lambda: nk.layernorm_bwd(x, x, g, mean, rstd, dresid=resid)),
            ("bias_grad_split N=3C", 2 * M * 3 * C * 4, lambda: nk.bias_grad_split(dyq)),
            ("bias_grad_split_gelu N=4C", 4 * M * F * 4, lambda: nk.bias_grad_split_gelu(dy3, pre3)),
            ("gelu_fwd_lo N=4C", 3 * M * F * 4, lambda: nk.gelu_fwd_lo(pre3)),
            ("split_lo [M, C]", 2 * M * C * 4, lambda: nk.split_lo(x)),
            ("cross_entropy", 2 * M * Vc * 4, lambda: nk.cross_entropy(logits, tgt)),
            ("embedding_fwd", 2 * M * C * 4, lambda: nk.embedding_fwd(tok, wte, wpe)),
            ("adamw_flat", 7 * P * 4, lambda: nk.adamw_flat(params, grads, mm, vv, [0, P], [0.0],
                                                           3e-4, 0.9, 0.95, 1e-8, 0.1, 0.05)),
        ]
        rows = []
        for name, nbytes, fn in cases:
            ms = _event_ms(torch, fn, args.reps)
            rows.append({"kernel": name, "us": ms * 1e3, "mb": nbytes / 1e6, "gbs": nbytes / ms / 1e6})
        out = {"case": "bw", "m_c_v": [M, C, Vc], "kernels": rows}
    nk.kernel_health()
    return out


def run_case(args):
    import torch

    fn = {"c1": case_c1, "c2": case_c2, "c3": case_c3, "c5": case_c5,
          "decode": case_decode, "lstm": case_lstm}.get(args.case, case_kernel)
    out = fn(args, torch)
    if out is not None:
        print(json.dumps(out), flush=True)


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.case != "step":
        run_case(args)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
