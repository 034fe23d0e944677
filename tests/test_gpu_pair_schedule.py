"""The CTA-pair GEMM's work schedule: in the dynamic order (engine 11, and a
data-parallel GPT backward) cluster c starts on tile c and then takes its
next tile (or stream-K run) from a per-launch counter when its producer is
ready for one; the fixed order (engine 0's GEMM calls, engine 10) hands the
same items out as cluster c takes items c, c + clusters, ....  Every item is computed
the same way whichever cluster takes it, so the two must agree bit for bit,
on plain, stream-K, split-K and transposed plans, with fewer tiles than
clusters, and over more launches than there are counter regions (each
launch's counter must be back at 0 for the next launch that uses it).
Reference: MatMul src/tensor.cpp:198-271.
"""
import numpy as np
import pytest
import torch

from neuralsuite_b200 import kernels as nk
from oracle import fp64
from tests._util import normal, rel_l2, rng

pytestmark = pytest.mark.gpu

FIXED = 10  # engine: the automatic plan, pair work in a fixed order
DYNAMIC = 11  # engine: the automatic plan, pair work from a per-launch counter


def dev(a, device):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32, device=device)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def operands(r, M, N, K, form):
    if form == "Y":  # X[M,K] . W[K,N]
        A, B = normal(r, (M, K)), normal(r, (K, N))
        return A, B, {}, fp64.matmul(A, B)
    if form == "dX":  # dY[M,K] . W[N,K]^T
        A, B = normal(r, (M, K)), normal(r, (N, K))
        return A, B, {"b_trans": True}, fp64.matmul(A, B.T)
    A, B = normal(r, (K, M)), normal(r, (K, N))  # dW: X[K,M]^T . dY[K,N]
    return A, B, {"a_trans": True}, fp64.matmul(A.T, B)


# The step's Linear shapes (whole waves of 256 x 256 / 192 / 128 pair tiles,
# stream-K tails on the N=768 products), a split-K head product, ragged edges,
# and a product with fewer tiles than clusters.
SHAPES = [(8192, 3072, 768), (8192, 2304, 768), (8192, 768, 3072), (8192, 256, 768),
          (256, 768, 8192), (6000, 1000, 2500), (512, 512, 512)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("form", ["Y", "dX", "dW"])
def test_dynamic_schedule_equals_fixed_order_bitwise(cuda, M, N, K, form):
    r = rng(11 * M + 5 * N + K + len(form))
    A, B, kw, want = operands(r, M, N, K, form)
    Ad, Bd = dev(A, cuda), dev(B, cuda)
    out = {}
    for engine in (DYNAMIC, FIXED, 0):
        nk.set_gemm_engine(engine)
        try:
            out[engine] = host(nk.gemm(Ad, Bd, **kw))
        finally:
            nk.set_gemm_engine(0)
    dyn, fixed = out[DYNAMIC], out[FIXED]
    assert rel_l2(dyn.astype(np.float64), want) < 5e-6, (form, M, N, K)
    assert np.array_equal(dyn.view(np.uint32), fixed.view(np.uint32)), (form, M, N, K)
    assert np.array_equal(out[0].view(np.uint32), fixed.view(np.uint32)), (form, M, N, K)
    nk.kernel_health()


def test_work_counters_return_to_zero_over_many_launches(cuda):
    """48 launches (three times round the 16 counter regions) of a stream-K
    product and a plain one, interleaved on one stream: every launch gives the
    first launch's bits, so no launch found its counter part-way."""
    nk.set_gemm_engine(DYNAMIC)
    try:
        _many_launches(cuda)
    finally:
        nk.set_gemm_engine(0)


def _many_launches(cuda):
    r = rng(2024)
    X, W = normal(r, (8192, 3072)), normal(r, (3072, 768))
    P, Q = normal(r, (8192, 768)), normal(r, (768, 3072))
    Xd, Wd, Pd, Qd = dev(X, cuda), dev(W, cuda), dev(P, cuda), dev(Q, cuda)
    first_a, first_b = host(nk.gemm(Xd, Wd)), host(nk.gemm(Pd, Qd))
    outs_a, outs_b = [], []
    for _ in range(24):
        outs_a.append(nk.gemm(Xd, Wd))
        outs_b.append(nk.gemm(Pd, Qd))
    for o in outs_a:
        assert np.array_equal(host(o).view(np.uint32), first_a.view(np.uint32))
    for o in outs_b:
        assert np.array_equal(host(o).view(np.uint32), first_b.view(np.uint32))
    nk.kernel_health()
