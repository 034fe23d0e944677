"""Small, self-contained kernel cases for profilers (ncu) and quick timing.

    python -m neuralsuite_b200.profile_cases gemm M N K [a_trans b_trans reps [engine [epilogue]]]
    python -m neuralsuite_b200.profile_cases attn B T H D [reps [engine]]
    python -m neuralsuite_b200.profile_cases ln ROWS DIM [reps]

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
    else:
        raise SystemExit(__doc__)
    nk.kernel_health()


if __name__ == "__main__":
    main(sys.argv[1:])
