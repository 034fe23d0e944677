"""LSTM and BiLSTM forward + backward against the reference's own LSTM /
BiLSTM (include/layers/lstm.h:320-664) through oracle.ref(): the output, the
input gradient and every parameter gradient at the north-star tolerance,
with float64 adjudication (oracle/fp64.lstm_fwd_bwd) of the elements that
miss.  Shapes include the reference test's small odd sizes, a hidden size
that is not a multiple of the per-CTA unit count, a single time step, and a
CRNN-sized sequence (T 64, batch 32, 256 features, 256 hidden).
"""
import numpy as np
import pytest
import torch

import oracle
from neuralsuite_b200 import kernels as nk
from oracle import fp64
from tests._util import close_report

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libnsref.so not built (needs the reference sources)")
    o = oracle.ref()
    o.set_threads(16)
    return o


def split(p, IN, H):
    a, b = 4 * H * IN, 4 * H * IN + 4 * H * H
    return p[:a].reshape(4 * H, IN), p[a:b].reshape(4 * H, H), p[b:b + 4 * H], p[b + 4 * H:b + 8 * H]


@pytest.mark.parametrize("T,B,IN,H", [(5, 3, 7, 4), (1, 2, 5, 9), (12, 4, 16, 13), (64, 32, 256, 256)])
@pytest.mark.parametrize("bidir", [False, True], ids=["lstm", "bilstm"])
def test_lstm_matches_reference(cuda, ref, T, B, IN, H, bidir):
    r = np.random.default_rng(T * 100 + B * 10 + IN + H + bidir)
    n1 = 4 * H * IN + 4 * H * H + 8 * H
    params = (r.standard_normal(n1 * (2 if bidir else 1)) / np.sqrt(H)).astype(np.float32)
    x = r.standard_normal((T, B, IN)).astype(np.float32)
    dout = r.standard_normal((T, B, (2 if bidir else 1) * H)).astype(np.float32)
    out_r, dx_r, g_r = ref.lstm(x, params, dout, H, bidir)
    out, dx, g = nk.lstm_fwd_bwd(torch.as_tensor(x, device="cuda"),
                                 torch.as_tensor(params, device="cuda"),
                                 torch.as_tensor(dout, device="cuda"), H, bidir)
    torch.cuda.synchronize()
    nk.kernel_health()
    lazy = {}

    def f64(i):
        if "v" not in lazy:
            if bidir:
                o6, dx6, g6 = fp64.bilstm_fwd_bwd(x, split(params[:n1], IN, H),
                                                  split(params[n1:], IN, H), dout)
            else:
                o6, dx6, g6 = fp64.lstm_fwd_bwd(x, *split(params, IN, H), dout)
            lazy["v"] = (o6, dx6, np.concatenate([a.reshape(-1) for a in g6]))
        return lazy["v"][i]

    for name, got, want, i in (("out", out, out_r, 0), ("dx", dx, dx_r, 1)):
        got = got.cpu().numpy()
        ok, info = close_report(got, want)
        if not ok:
            ok, info = close_report(got, want, f64(i))
        assert ok, (name, info)
    # every parameter gradient tensor on its own (the float64 slack is per tensor)
    g = g.cpu().numpy()
    sizes = [4 * H * IN, 4 * H * H, 4 * H, 4 * H] * (2 if bidir else 1)
    names = ["w_ih", "w_hh", "b_ih", "b_hh"] * 2
    off = 0
    for name, n in zip(names, sizes):
        sl = slice(off, off + n)
        ok, info = close_report(g[sl], g_r[sl])
        if not ok:
            ok, info = close_report(g[sl], g_r[sl], f64(2)[sl])
        assert ok, (name, off, info)
        off += n


def test_lstm_is_deterministic(cuda):
    r = np.random.default_rng(9)
    T, B, IN, H = 20, 8, 32, 48
    n1 = 4 * H * IN + 4 * H * H + 8 * H
    p = torch.as_tensor((r.standard_normal(2 * n1) * 0.1).astype(np.float32), device="cuda")
    x = torch.as_tensor(r.standard_normal((T, B, IN)).astype(np.float32), device="cuda")
    d = torch.as_tensor(r.standard_normal((T, B, 2 * H)).astype(np.float32), device="cuda")
    a = nk.lstm_fwd_bwd(x, p, d, H, True)
    b = nk.lstm_fwd_bwd(x, p, d, H, True)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_whole_sequence_recurrence_equals_per_step_launches(cuda):
    """The cooperative whole-sequence kernels and the per-step kernels do the
    same sums in the same order: every output bit-identical."""
    T, B, IN, H = 24, 8, 32, 64
    r = np.random.default_rng(13)
    n1 = 4 * H * IN + 4 * H * H + 8 * H
    p = torch.as_tensor((r.standard_normal(2 * n1) / 8).astype(np.float32), device="cuda")
    x = torch.as_tensor(r.standard_normal((T, B, IN)).astype(np.float32), device="cuda")
    d = torch.as_tensor(r.standard_normal((T, B, 2 * H)).astype(np.float32), device="cuda")
    try:
        whole = [t.cpu().numpy() for t in nk.lstm_fwd_bwd(x, p, d, H, True)]
        nk.lstm_set_engine(1)
        steps = [t.cpu().numpy() for t in nk.lstm_fwd_bwd(x, p, d, H, True)]
    finally:
        nk.lstm_set_engine(0)
    nk.kernel_health()
    for a, b in zip(whole, steps):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
