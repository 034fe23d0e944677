"""The GEMM's stream-K tail (CTA-pair tiles): shapes whose tiles leave a
part-filled last wave share the leftover tiles' k-blocks among all pairs and
sum the partial tiles in k order.  Checked against float64 with the MatMul
sweep's bar, against the planner's plan without the tail (engine 9), for
every epilogue, and for run-to-run determinism.  Reference: MatMul
src/tensor.cpp:198-271 (the product every Linear layer runs).
"""
import numpy as np
import pytest
import torch

from neuralsuite_b200 import _lib
from neuralsuite_b200 import kernels as nk
from oracle import fp64
from tests._util import normal, rel_l2, rng

pytestmark = pytest.mark.gpu

NO_TAIL = 9  # engine: the automatic plan with the stream-K tail switched off


def dev(a, device):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32, device=device)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def check64(got, want, what):
    """relL2 <= 5e-6 and 1e-4 relative wherever |want| >= 0.1 rms (the sweep's bar)."""
    g = got.astype(np.float64)
    e = rel_l2(g, want)
    rms = np.sqrt(np.mean(want * want))
    big = np.abs(want) >= 0.1 * rms
    worst = float((np.abs(g - want)[big] / np.abs(want[big])).max())
    assert e < 5e-6 and worst < 1e-4, (what, e, worst)


def run(engine, fn):
    nk.set_gemm_engine(engine)
    try:
        return host(fn())
    finally:
        nk.set_gemm_engine(0)


# (M, N, K) of products the planner runs with a tail (one whole wave of
# 256 x 256 pair tiles, then 22-54 leftover tiles): the step's mlp_proj
# forward and mlp_fc / c_attn input-gradient shapes, and ragged shapes (K not
# a multiple of the 32-wide k-block, edges not a multiple of the tile; stored
# rows stay a multiple of 4 floats, which the pair tiles' TMA copies need).
SHAPES = [(8192, 768, 3072), (8192, 768, 2304), (6000, 1000, 2500), (9000, 700, 3000),
          (10000, 600, 2052)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("form", ["Y", "dX", "dW"])
def test_stream_k_matches_float64_and_plain_plan(cuda, M, N, K, form):
    r = rng(M + 3 * N + 7 * K)
    if form == "Y":  # X[M,K] . W[K,N]
        A, B = normal(r, (M, K)), normal(r, (K, N))
        fn = lambda: nk.gemm(dev(A, cuda), dev(B, cuda))
        want = fp64.matmul(A, B)
    elif form == "dX":  # dY[M,K] . W[N,K]^T
        A, B = normal(r, (M, K)), normal(r, (N, K))
        fn = lambda: nk.gemm(dev(A, cuda), dev(B, cuda), b_trans=True)
        want = fp64.matmul(A, B.T)
    else:  # X[K,M]^T . dY[K,N]
        A, B = normal(r, (K, M)), normal(r, (K, N))
        fn = lambda: nk.gemm(dev(A, cuda), dev(B, cuda), a_trans=True)
        want = fp64.matmul(A.T, B)
    sk = run(0, fn)
    check64(sk, want, f"{form} {M}x{N}x{K} stream-K")
    again = run(0, fn)
    assert np.array_equal(sk.view(np.uint32), again.view(np.uint32)), "stream-K not deterministic"
    plain = run(NO_TAIL, fn)
    check64(plain, want, f"{form} {M}x{N}x{K} plain")
    # The tail sums k-runs in another grouping than whole tiles do: a bit-for-bit
    # match would mean the tail never ran.
    assert not np.array_equal(sk.view(np.uint32), plain.view(np.uint32)), "no stream-K tail taken"
    nk.kernel_health()


@pytest.mark.parametrize("M,N,K", [(8192, 768, 2304), (6000, 1000, 2500)])
def test_stream_k_epilogues(cuda, M, N, K):
    """Bias, bias+GELU (both outputs), bias+residual, GELU backward, beta=1
    and the output's lo part, each through the warp that completes a tail
    tile, against the same epilogue on the plain plan."""
    r = rng(M * 5 + N + K)
    X, W = normal(r, (M, K)), normal(r, (K, N), 0.05)
    b, R = normal(r, N), normal(r, (M, N))
    Xd, Wd, bd, Rd = dev(X, cuda), dev(W, cuda), dev(b, cuda), dev(R, cuda)
    base64 = fp64.matmul(X, W)
    outs = {}
    for engine in (0, NO_TAIL):
        nk.set_gemm_engine(engine)
        try:
            o = {}
            o["bias"] = host(nk.gemm(Xd, Wd, epilogue=_lib.EPI_BIAS, bias=bd))
            yc, yg = nk.gemm(Xd, Wd, epilogue=_lib.EPI_BIAS_GELU, bias=bd)
            o["gelu_pre"], o["gelu"] = host(yc), host(yg)
            o["resid"] = host(nk.gemm(Xd, Wd, epilogue=_lib.EPI_BIAS_RESID, bias=bd, aux=Rd))
            o["gelu_bwd"] = host(nk.gemm(Xd, Wd, epilogue=_lib.EPI_GELU_BWD, aux=Rd))
            acc = dev(R, cuda)
            nk.gemm(Xd, Wd, out=acc, beta=1.0)
            o["beta1"] = host(acc)
            lo = torch.empty(M, N, device=cuda)
            y = nk.gemm(Xd, Wd, epilogue=_lib.EPI_BIAS, bias=bd, out_lo=lo)
            o["lo_y"], o["lo"] = host(y), host(lo)
            outs[engine] = o
        finally:
            nk.set_gemm_engine(0)
    sk, plain = outs[0], outs[NO_TAIL]
    check64(sk["bias"], base64 + b, "bias")
    check64(sk["gelu_pre"], base64 + b, "bias_gelu pre")
    check64(sk["gelu"], fp64.gelu(base64 + b), "bias_gelu post")
    check64(sk["resid"], R + (base64 + b), "bias_resid")
    check64(sk["gelu_bwd"], base64 * fp64.gelu_grad(R), "gelu_bwd")
    check64(sk["beta1"], R + base64, "beta1")
    hi = (sk["lo_y"].view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    assert np.array_equal(sk["lo"].view(np.uint32), (sk["lo_y"] - hi).view(np.uint32)), "out_lo"
    for k in sk:
        tol = 1e-5 + 1e-4 * np.abs(plain[k])
        assert np.mean(np.abs(sk[k] - plain[k]) <= tol) > 0.999, k
    nk.kernel_health()
