"""Small, self-contained kernel cases for profilers (ncu) and quick timing.

    python -m neuralsuite_b200.profile_cases gemm M N K [a_trans b_trans reps [engine [epilogue]]]
    python -m neuralsuite_b200.profile_cases attn B T H D [reps [engine]]
    python -m neuralsuite_b200.profile_cases ln ROWS DIM [reps]
    python -m neuralsuite_b200.profile_cases bw [M C V]

`bw` runs each bandwidth-bound kernel of a GPT training step once at the
step's shapes (M = B*T rows, C = width, V = vocab; default 8192 768 256) and
prints the CUDA-event time and the algorithmic bytes of each launch.

Each case allocates its operands once (seeded normal data), runs the kernel
`reps` times on the current stream (default 3) and prints the CUDA-event time
of the last launch.  Sizes are chosen by the caller so that a profiler capture
stays small (a few GB on the device at most).
"""
from __future__ import annotations

import sys

import torch

from . import kernels as nk


def _time(fn, reps):
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(reps - 1):
        fn()
    s.record()
    fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e)


def main(argv):
    torch.manual_seed(0)
    dev = torch.device("cuda")
    case = argv[0]
    if case == "gemm":
        M, N, K = (int(x) for x in argv[1:4])
        at = int(argv[4]) if len(argv) > 4 else 0
        bt = int(argv[5]) if len(argv) > 5 else 0
        reps = int(argv[6]) if len(argv) > 6 else 3
        if len(argv) > 7:
            nk.set_gemm_engine(int(argv[7]))
        epi = int(argv[8]) if len(argv) > 8 else 0
        A = torch.randn((K, M) if at else (M, K), device=dev)
        B = torch.randn((N, K) if bt else (K, N), device=dev)
        out = torch.empty(M, N, device=dev)
        bias = torch.randn(N, device=dev)
        aux = torch.randn(M, N, device=dev)
        kw = {}
        if epi in (1, 2, 3):
            kw["bias"] = bias
        if epi in (3, 4):
            kw["aux"] = aux
        if epi == 2:
            kw["aux_out"] = torch.empty(M, N, device=dev)
        ms = _time(lambda: nk.gemm(A, B, a_trans=bool(at), b_trans=bool(bt), out=out, epilogue=epi,
                                   **kw), reps)
        print(f"gemm {M}x{N}x{K} at={at} bt={bt} epi={epi}: {ms:.4f} ms, "
              f"{2 * M * N * K / ms / 1e9:.1f} TFLOP/s")
    elif case == "attn":
        Bb, T, H, D = (int(x) for x in argv[1:5])
        reps = int(argv[5]) if len(argv) > 5 else 3
        qkv = torch.randn(Bb * T, 3 * H * D, device=dev)
        dout = torch.randn(Bb * T, H * D, device=dev)
        engines = [int(argv[6])] if len(argv) > 6 else [0, 1]
        for eng in engines:
            nk.attn_set_engine(eng)
            out, lse = nk.attn_fwd(qkv, Bb, T, H, D)
            f = _time(lambda: nk.attn_fwd(qkv, Bb, T, H, D), reps)
            b = _time(lambda: nk.attn_bwd(qkv, out, dout, lse, Bb, T, H, D), reps)
            name = "simt" if eng else "auto"
            print(f"attention[{name}] B={Bb} T={T} H={H} D={D}: fwd {f:.3f} ms, bwd {b:.3f} ms")
        nk.attn_set_engine(0)
    elif case == "ln":
        rows, dim = int(argv[1]), int(argv[2])
        reps = int(argv[3]) if len(argv) > 3 else 3
        x = torch.randn(rows, dim, device=dev)
        g = torch.ones(dim, device=dev)
        b = torch.zeros(dim, device=dev)
        y, m, r = nk.layernorm_fwd(x, g, b)
        f = _time(lambda: nk.layernorm_fwd(x, g, b), reps)
        bw = _time(lambda: nk.layernorm_bwd(x, x, g, m, r, dresid=x), reps)
        print(f"layernorm {rows}x{dim}: fwd {f:.4f} ms, bwd {bw:.4f} ms")
    elif case == "bw":
        M, C, V = (int(x) for x in argv[1:4]) if len(argv) > 3 else (8192, 768, 256)
        F = 4 * C
        r = lambda *shape: torch.randn(*shape, device=dev)
        x, resid, raw = r(M, C), r(M, C), r(M, C)
        g, b, bias = r(C), r(C), r(C)
        dy3, pre3 = r(M, F), r(M, F)
        dyq = r(M, 3 * C)
        logits = r(M, V)
        tgt = torch.randint(0, V, (M,), device=dev, dtype=torch.int32)
        tok = torch.randint(0, V, (M // 1024, 1024), device=dev, dtype=torch.int32)
        wte, wpe = r(V, C), r(1024, C)
        P = 86_039_040
        params, grads, m, v = r(P), r(P), torch.zeros(P, device=dev), torch.zeros(P, device=dev)
        _, _, _, mean, rstd = nk.layernorm_fwd_ex(x, g, b)
        B4 = 4  # bytes per float
        cases = [
            ("ln_fwd_ex (resid + LayerNorm + lo)", (5 * M * C + 2 * M) * B4,
             lambda: nk.layernorm_fwd_ex(raw, g, b, bias=bias, resid=resid)),
            ("ln_bwd (+ dresid)", 4 * M * C * B4, lambda: nk.layernorm_bwd(x, x, g, mean, rstd, dresid=resid)),
            ("bias_grad_split N=3C", 2 * M * 3 * C * B4, lambda: nk.bias_grad_split(dyq)),
            ("bias_grad_split_gelu N=4C", 4 * M * F * B4, lambda: nk.bias_grad_split_gelu(dy3, pre3)),
            ("gelu_fwd_lo N=4C", 3 * M * F * B4, lambda: nk.gelu_fwd_lo(pre3)),
            ("split_lo [M, C]", 2 * M * C * B4, lambda: nk.split_lo(x)),
            ("cross_entropy", 2 * M * V * B4, lambda: nk.cross_entropy(logits, tgt)),
            ("embedding_fwd", 2 * M * C * B4, lambda: nk.embedding_fwd(tok, wte, wpe)),
            ("adamw_flat", 7 * P * B4, lambda: nk.adamw_flat(params, grads, m, v, [0, P], [0.0],
                                                               3e-4, 0.9, 0.95, 1e-8, 0.1, 0.05)),
        ]
        for name, nbytes, fn in cases:
            ms = _time(fn, 2)
            print(f"{name:36s} {ms * 1000:8.1f} us  {nbytes / 1e6:8.1f} MB  {nbytes / ms / 1e6:7.0f} GB/s")
    else:
        raise SystemExit(__doc__)
    nk.kernel_health()


if __name__ == "__main__":
    main(sys.argv[1:])
