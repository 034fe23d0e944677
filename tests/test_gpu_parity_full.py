"""Full-size parity against the NeuralSuite reference itself (oracle.ref(),
its own src/tensor.cpp and headers compiled by oracle/Makefile, run on all
host cores).

Tolerance (north star): every float output within
|x - ref| <= 1e-5 + 1e-4*|ref| of the fp32 reference, element by element;
only the elements that miss are adjudicated against the float64
restatement (tests/_util.close_report), which is therefore computed only
when some element misses.

* the 12-layer / 768-wide GPT training step at T=1024, B=8 (loss, logits,
  all 148 gradients, then the parameters after one AdamW step);
* the MatMul sweep (Y, dX, dW at (512,128,512), (8192,768,3072),
  (8192,3072,768), (16384,1024,4096));
* the MultiHeadAttention layer at B=8, T=1024, 12 heads, n_embd 768 composed
  through the C ABI (c_attn, causal attention, c_proj; forward output, input
  gradient and the four projection gradients), every batch.
"""
import os

import numpy as np
import pytest
import torch

import oracle
from neuralsuite_b200 import GPTConfig, GPTModel, _lib, param_shapes
from neuralsuite_b200 import kernels as nk
from oracle import fp64
from tests._util import close_report, gpt_init, normal, rng

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


@pytest.fixture(scope="module")
def ref():
    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libnsref.so not built (needs the reference sources)")
    o = oracle.ref()
    o.set_threads(os.cpu_count() or 1)
    return o


def dev(a, device):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32, device=device)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


class Lazy64:
    """float64 restatement computed on first use (only when an element misses)."""

    def __init__(self, fn):
        self.fn, self.val = fn, None

    def get(self):
        if self.val is None:
            self.val = self.fn()
        return self.val


def check(tag, got, want32, lazy64=None, pick=None):
    ok, info = close_report(got, want32)
    if not ok and lazy64 is not None:
        t = lazy64.get()
        ok, info = close_report(got, want32, pick(t) if pick else t)
    print(f"{tag}: {info}")
    assert ok, (tag, info)
    return info


# ----------------------------------------------------------- GPT 12L / 768

def test_config4_step_vs_reference(cuda, ref):
    """12 layers, n_embd 768, 12 heads, T=1024, 8 sequences, vocab 256, the
    reference's initialisation, uniform byte tokens: the device step against
    GPTModel::Forward -> CrossEntropyLoss -> GPTModel::Backward
    (include/gpt.h:192-272) and one AdamW::Step (include/optimizers.h:206-234)
    of the reference on the same weights and tokens."""
    V, block, L, H, C, B, T = 256, 1024, 12, 12, 768, 8, 1024
    cfg = GPTConfig(V, block, L, H, C)
    r = rng(2024)
    flat = gpt_init(param_shapes(cfg), r, ln_noise=0.05)
    idx = r.integers(0, V, (B, T)).astype(np.float32)
    tgt = r.integers(0, V, B * T).astype(np.float32)

    g = ref.gpt(V, block, L, H, C)
    assert g.num_params() == 86_039_040
    g.set_params(flat)
    rl, rlog = g.fwd_bwd(idx, tgt)
    rgr = g.get_grads()

    m = GPTModel(cfg, max_batch=B)
    assert m.n_params == 86_039_040 and m.n_tensors == 148
    m.set_params(flat)
    loss, logits = m.fwd_bwd(idx, tgt)
    grads = m.get_grads()
    nk.kernel_health()

    lazy = Lazy64(lambda: fp64.gpt_fwd_bwd(flat, idx, tgt, V, block, L, H, C, keep_probs=False))
    check("loss", np.array([loss]), np.array([rl], np.float32), lazy,
          lambda t: np.array([t[0]]))
    check("logits", logits, rlog, lazy, lambda t: t[1])
    offs = [m.tensor_offset(i) for i in range(m.n_tensors)] + [m.n_params]
    worst = 0.0
    for i in range(m.n_tensors):
        a, b = offs[i], offs[i + 1]
        info = check(f"grad[{i}]", grads[a:b], rgr[a:b], lazy, lambda t, a=a, b=b: t[2][a:b])
        worst = max(worst, info["max_abs"])
    print("worst |grad - ref|:", worst)

    lr = 3e-4
    g.adamw_init(lr)
    g.adamw_step()
    m.adamw_init(lr)
    m.adamw_step()
    p_ref = g.get_params().astype(np.float64)
    p_got = m.get_params().astype(np.float64)
    err = np.abs(p_got - p_ref)
    tight = err <= 1e-5 + 1e-4 * np.abs(p_ref)
    # The first Adam step moves a parameter by lr * m/sqrt(v) = +-lr for any
    # gradient away from zero; where the gradient itself is at rounding level
    # the sign can differ, so all parameters are within 2*lr and nearly all
    # within the step tolerance.
    print("params after AdamW: within tol", float(tight.mean()), "max err", float(err.max()))
    assert tight.mean() >= 0.999, float(tight.mean())
    assert err.max() <= 2 * lr + 1e-6, float(err.max())


# ----------------------------------------------------------- MatMul sweep

SWEEP = [(512, 128, 512), (8192, 768, 3072), (8192, 3072, 768), (16384, 1024, 4096)]


@pytest.mark.parametrize("M,K,N", SWEEP)
def test_matmul_sweep_vs_reference(cuda, ref, M, K, N):
    """Y = X.W, dX = dY.W^T and dW = X^T.dY (Linear::Forward/Backward,
    include/layers/linear.h:59-116) against the reference's MatMul
    (src/tensor.cpp:198-271) on its explicit Transpose copies (275-288)."""
    r = rng(M + 3 * K + 7 * N)
    X, W, dY = normal(r, (M, K)), normal(r, (K, N)), normal(r, (M, N))
    Xd, Wd, dYd = dev(X, cuda), dev(W, cuda), dev(dY, cuda)
    cases = (
        ("Y", lambda: nk.gemm(Xd, Wd), lambda: ref.matmul(X, W), lambda: fp64.matmul(X, W)),
        ("dX", lambda: nk.gemm(dYd, Wd, b_trans=True), lambda: ref.matmul(dY, W.T.copy()),
         lambda: fp64.matmul(dY, W.T)),
        ("dW", lambda: nk.gemm(Xd, dYd, a_trans=True), lambda: ref.matmul(X.T.copy(), dY),
         lambda: fp64.matmul(X.T, dY)),
    )
    for name, got, want, want64 in cases:
        check(f"{name} {M}x{K}x{N}", host(got()), want(), Lazy64(want64))
    nk.kernel_health()


# ------------------------------------------------- MultiHeadAttention layer

def mha_device(x, wa, ba, wp, bp, dout, B, T, H, C):
    """The layer composed from the C ABI as MultiHeadAttention::Forward /
    ::Backward order their steps (include/layers/attention.h:350-467):
    qkv = x.Wa + ba; core; y = att.Wp + bp; then dWp = att^T.dy, dbp,
    datt = dy.Wp^T, core backward, dWa = x^T.dqkv, dba, dx = dqkv.Wa^T."""
    D = C // H
    qkv = nk.gemm(x, wa, epilogue=_lib.EPI_BIAS, bias=ba)
    att, lse = nk.attn_fwd(qkv, B, T, H, D)
    y = nk.gemm(att, wp, epilogue=_lib.EPI_BIAS, bias=bp)
    g_wp = nk.gemm(att, dout, a_trans=True)
    g_bp = nk.bias_grad(dout)
    datt = nk.gemm(dout, wp, b_trans=True)
    dqkv = nk.attn_bwd(qkv, att, datt, lse, B, T, H, D)
    g_wa = nk.gemm(x, dqkv, a_trans=True)
    g_ba = nk.bias_grad(dqkv)
    dx = nk.gemm(dqkv, wa, b_trans=True)
    return y, dx, [g_wa, g_ba, g_wp, g_bp]


def mha_fp64(x, wa, ba, wp, bp, dout, B, T, H, C):
    D = C // H
    x64 = fp64.f64(x)
    qkv = x64 @ fp64.f64(wa) + fp64.f64(ba)
    att, p = fp64.attention_fwd(qkv, B, T, H, D)
    y = att @ fp64.f64(wp) + fp64.f64(bp)
    d = fp64.f64(dout)
    g_wp, g_bp = att.T @ d, d.sum(0)
    datt = d @ fp64.f64(wp).T
    dqkv = fp64.attention_bwd(qkv, p, datt, B, T, H, D)
    del p
    return y, dqkv @ fp64.f64(wa).T, [x64.T @ dqkv, dqkv.sum(0), g_wp, g_bp]


def test_mha_layer_vs_reference(cuda, ref):
    """B=8, T=1024, 12 heads, n_embd 768 (head size 64): x and the upstream
    gradient N(0,1), projection weights N(0,0.02) and biases N(0,0.02)."""
    B, T, H, C = 8, 1024, 12, 768
    r = rng(3108)
    x = normal(r, (B * T, C))
    dout = normal(r, (B * T, C))
    wa, ba = normal(r, (C, 3 * C), 0.02), normal(r, 3 * C, 0.02)
    wp, bp = normal(r, (C, C), 0.02), normal(r, C, 0.02)
    y_r, dx_r, g_r = ref.mha(B, T, C, H, wa, ba, wp, bp, x.reshape(B, T, C), dout.reshape(B, T, C))
    y, dx, g = mha_device(dev(x, cuda), dev(wa, cuda), dev(ba, cuda), dev(wp, cuda), dev(bp, cuda),
                          dev(dout, cuda), B, T, H, C)
    nk.kernel_health()
    lazy = Lazy64(lambda: mha_fp64(x, wa, ba, wp, bp, dout, B, T, H, C))
    check("y", host(y), y_r.reshape(B * T, C), lazy, lambda t: t[0])
    check("dx", host(dx), dx_r.reshape(B * T, C), lazy, lambda t: t[1])
    for i, name in enumerate(["c_attn.W", "c_attn.b", "c_proj.W", "c_proj.b"]):
        check(name, host(g[i]), g_r[i], lazy, lambda t, i=i: t[2][i])
