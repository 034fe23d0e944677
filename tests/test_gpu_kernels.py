"""Kernel-level parity: each C-ABI entry point against the oracle on seeded inputs.

fp32 outputs must satisfy |x - ref| <= 1e-5 + 1e-4*|ref| against the fp32 CPU
oracle (bit-identical to the reference), with float64 adjudication of misses
(tests/_util.close_report); integer/index work and the order-preserving
kernels (embedding backward, AdamW) must be bit-exact.
"""
import numpy as np
import pytest
import torch

from neuralsuite_b200 import _lib
from neuralsuite_b200 import kernels as nk
from oracle import fp64
from tests._util import assert_close, normal, rel_l2, rng

pytestmark = pytest.mark.gpu


def dev(a, device, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device=device)


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


# ------------------------------------------------------------------- GEMM

SMALL = [(512, 128, 512), (512, 128, 384), (300, 200, 100), (128, 64, 256), (8, 8, 8)]


@pytest.mark.parametrize("M,K,N", SMALL)
def test_gemm_three_forms_small(cuda, port, M, K, N):
    """Y = X.W, dX = dY.W^T, dW = X^T.dY against MatMul on explicit transposes."""
    r = rng(M * 7 + K * 3 + N)
    X, W, dY = normal(r, (M, K)), normal(r, (K, N)), normal(r, (M, N))
    Xd, Wd, dYd = dev(X, cuda), dev(W, cuda), dev(dY, cuda)
    y = host(nk.gemm(Xd, Wd))
    assert_close(y, port.matmul(X, W), fp64.matmul(X, W), what="Y")
    dx = host(nk.gemm(dYd, Wd, b_trans=True))
    assert_close(dx, port.matmul(dY, W.T.copy()), fp64.matmul(dY, W.T), what="dX")
    dw = host(nk.gemm(Xd, dYd, a_trans=True))
    assert_close(dw, port.matmul(X.T.copy(), dY), fp64.matmul(X.T, dY), what="dW")


def test_gemm_known_answer(cuda):
    """MatMul KAT of test_suite.cpp:97-118 (2x3 . 3x2 = [31, 19, 85, 55])."""
    A = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    B = np.array([[7, 8], [9, 1], [2, 3]], np.float32)
    c = host(nk.gemm(dev(A, cuda), dev(B, cuda)))
    np.testing.assert_array_equal(c, np.array([[31, 19], [85, 55]], np.float32))


def test_gemm_tf32_split_recovers_fp32(cuda):
    """Operands with all 24 mantissa bits set: a single-pass TF32 product would
    lose ~1e-3 relative; 3xTF32 must be within a few fp32 ulps."""
    M = N = 128
    Kd = 256
    r = rng(11)
    A = (1.0 + r.random((M, Kd)) * 2 ** -10).astype(np.float32)  # low mantissa bits only
    B = (1.0 + r.random((Kd, N)) * 2 ** -10).astype(np.float32)
    c = host(nk.gemm(dev(A, cuda), dev(B, cuda)))
    exact = fp64.matmul(A, B)
    rel = np.abs(c - exact) / exact
    assert rel.max() < 2e-6, rel.max()


FULL = [(8192, 768, 3072), (8192, 3072, 768), (16384, 1024, 4096)]


@pytest.fixture(params=[0, 2, 3, 4, 5, 6, 7],
                ids=["auto", "inkernel", "pair", "wide", "widerows", "pair192", "pair128"])
def gemm_engine(request):
    nk.set_gemm_engine(request.param)
    yield request.param
    nk.set_gemm_engine(0)


@pytest.mark.slow
@pytest.mark.parametrize("M,K,N", FULL)
def test_gemm_sweep_full(cuda, gemm_engine, M, K, N):
    """The MatMul sweep shapes: every form against float64.  Relative L2
    error <= 5e-6 (the reference's own bar for its fast-vs-literal attention
    is 1e-5, test_suite.cpp:3148-3150; an fp32 k-sequential loop lands near
    1e-6 here) and, per element, within 1e-4 relative of the float64 value
    wherever |value| >= 0.1 * rms (smaller values carry the same absolute
    rounding as any fp32 accumulation of K products).  Every tcgen05 kernel:
    the planner's choice, in-kernel operand split, CTA-pair tiles, 128 x 256
    tiles."""
    r = rng(M + K + N)
    X, W, dY = normal(r, (M, K)), normal(r, (K, N)), normal(r, (M, N))
    Xd, Wd, dYd = dev(X, cuda), dev(W, cuda), dev(dY, cuda)
    for name, got, ref in (
        ("Y", lambda: nk.gemm(Xd, Wd), lambda: fp64.matmul(X, W)),
        ("dX", lambda: nk.gemm(dYd, Wd, b_trans=True), lambda: fp64.matmul(dY, W.T)),
        ("dW", lambda: nk.gemm(Xd, dYd, a_trans=True), lambda: fp64.matmul(X.T, dY)),
    ):
        g = host(got()).astype(np.float64)
        t = ref()
        e = rel_l2(g, t)
        rms = np.sqrt(np.mean(t * t))
        big = np.abs(t) >= 0.1 * rms
        worst = float((np.abs(g - t)[big] / np.abs(t[big])).max())
        print(f"{name} {M}x{K}x{N}: relL2 {e:.2e} worst rel (|ref|>=0.1 rms) {worst:.2e}")
        assert e < 5e-6, (name, e)
        assert worst < 1e-4, (name, worst)
        del g, t
    nk.kernel_health()


def test_gemm_engines_agree_and_epilogues(cuda, port):
    M, Kd, N = 640, 256, 384
    r = rng(5)
    X, W = normal(r, (M, Kd)), normal(r, (Kd, N), 0.05)
    b, R = normal(r, N), normal(r, (M, N))
    Xd, Wd, bd, Rd = dev(X, cuda), dev(W, cuda), dev(b, cuda), dev(R, cuda)
    base = port.matmul(X, W)
    base64 = fp64.matmul(X, W)
    for engine in (0, 1, 2, 3, 4, 5, 6, 7):
        nk.set_gemm_engine(engine)
        try:
            y = host(nk.gemm(Xd, Wd, epilogue=_lib.EPI_BIAS, bias=bd))
            assert_close(y, base + b, base64 + b, what=f"bias e{engine}")
            yc, yg = nk.gemm(Xd, Wd, epilogue=_lib.EPI_BIAS_GELU, bias=bd)
            assert_close(host(yc), base + b, base64 + b, what=f"bias_gelu pre e{engine}")
            assert_close(host(yg), port.gelu_fwd(base + b), fp64.gelu(base64 + b),
                         what=f"bias_gelu post e{engine}")
            yr = host(nk.gemm(Xd, Wd, epilogue=_lib.EPI_BIAS_RESID, bias=bd, aux=Rd))
            assert_close(yr, R + (base + b), R + (base64 + b), what=f"resid e{engine}")
            yb = host(nk.gemm(Xd, Wd, epilogue=_lib.EPI_GELU_BWD, aux=Rd))
            assert_close(yb, port.gelu_bwd(base, R), base64 * fp64.gelu_grad(R),
                         what=f"gelu_bwd e{engine}")
            acc = dev(R, cuda)
            nk.gemm(Xd, Wd, out=acc, beta=1.0)
            assert_close(host(acc), R + base, R + base64, what=f"beta1 e{engine}")
        finally:
            nk.set_gemm_engine(0)


def test_split_lo_is_exact(cuda):
    """ns_split_lo: x - trunc_tf32(x), bit for bit (hi + lo == x)."""
    x = normal(rng(21), (300, 772)) * np.float32(37.0)
    lo = host(nk.split_lo(dev(x, cuda)))
    hi = (x.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    assert np.array_equal(lo.view(np.uint32), (x - hi).view(np.uint32))
    assert np.array_equal((hi + lo).view(np.uint32), x.view(np.uint32))


@pytest.mark.parametrize("M,K,N,at,bt", [(8192, 768, 3072, 0, 0), (8192, 3072, 768, 0, 1),
                                         (768, 8192, 3072, 1, 0), (300, 200, 1000, 0, 0),
                                         (8192, 768, 256, 0, 1)])
def test_gemm_lo_equals_gemm_bitwise(cuda, M, K, N, at, bt):
    """ns_gemm_lo with caller-made lo copies (both, either, none) gives the
    same bits as ns_gemm: same kernel, same operand split."""
    r = rng(M + K + N + at + bt)
    A = dev(normal(r, (K, M) if at else (M, K)), cuda)
    B = dev(normal(r, (N, K) if bt else (K, N)), cuda)
    ref = host(nk.gemm(A, B, a_trans=bool(at), b_trans=bool(bt))).view(np.uint32)
    alo, blo = nk.split_lo(A), nk.split_lo(B)
    for a_lo, b_lo in ((alo, blo), (alo, None), (None, blo)):
        got = host(nk.gemm(A, B, a_trans=bool(at), b_trans=bool(bt), a_lo=a_lo, b_lo=b_lo))
        assert np.array_equal(got.view(np.uint32), ref)
    nk.kernel_health()


def test_bias_grad_split_matches_parts_bitwise(cuda):
    """ns_bias_grad_split = ns_bias_grad + ns_split_lo, bit for bit."""
    dY = dev(normal(rng(31), (8192, 768)), cuda)
    db, lo = nk.bias_grad_split(dY)
    assert np.array_equal(host(db).view(np.uint32), host(nk.bias_grad(dY)).view(np.uint32))
    assert np.array_equal(host(lo).view(np.uint32), host(nk.split_lo(dY)).view(np.uint32))


def test_bias_grad_split_gelu_matches_parts_bitwise(cuda):
    """ns_bias_grad_split_gelu = ns_gelu_bwd, then ns_bias_grad + ns_split_lo, bit for bit."""
    dpost = dev(normal(rng(32), (4096, 3072)), cuda)
    pre = dev(normal(rng(33), (4096, 3072), std=2.0), cuda)
    want = nk.gelu_bwd(dpost, pre)
    got, db, lo = nk.bias_grad_split_gelu(dpost.clone(), pre)
    assert np.array_equal(host(got).view(np.uint32), host(want).view(np.uint32))
    assert np.array_equal(host(db).view(np.uint32), host(nk.bias_grad(want)).view(np.uint32))
    assert np.array_equal(host(lo).view(np.uint32), host(nk.split_lo(want)).view(np.uint32))


@pytest.mark.parametrize("M,N,K", [(8192, 2304, 768), (8192, 3072, 768), (768, 768, 8192),
                                   (300, 200, 100), (256, 264, 2048)])
@pytest.mark.parametrize("epi", [_lib.EPI_STORE, _lib.EPI_BIAS, _lib.EPI_BIAS_GELU,
                                 _lib.EPI_BIAS_RESID, _lib.EPI_GELU_BWD])
def test_gemm_out_lo_is_split_of_output(cuda, M, N, K, epi):
    """ns_gemm_lo_out: same C (and aux_out) as ns_gemm_lo, plus out_lo = split of the activation."""
    r = rng(M + N + K + epi)
    A = dev(normal(r, (M, K)), cuda)
    B = dev(normal(r, (K, N)), cuda)
    bias = dev(normal(r, (N,)), cuda)
    aux = dev(normal(r, (M, N)), cuda) if epi in (_lib.EPI_BIAS_RESID, _lib.EPI_GELU_BWD) else None
    a_lo, b_lo = nk.split_lo(A), nk.split_lo(B)
    kw = dict(epilogue=epi, bias=bias if epi in (_lib.EPI_BIAS, _lib.EPI_BIAS_GELU, _lib.EPI_BIAS_RESID) else None,
              aux=aux, a_lo=a_lo, b_lo=b_lo)
    want = nk.gemm(A, B, **kw)
    lo = torch.empty((M, N), device=cuda)
    got = nk.gemm(A, B, out_lo=lo, **kw)
    if epi == _lib.EPI_BIAS_GELU:
        (wc, wg), (gc, gg) = want, got
        assert np.array_equal(host(gc).view(np.uint32), host(wc).view(np.uint32))
        assert np.array_equal(host(gg).view(np.uint32), host(wg).view(np.uint32))
        act = wg
    else:
        assert np.array_equal(host(got).view(np.uint32), host(want).view(np.uint32))
        act = want
    assert np.array_equal(host(lo).view(np.uint32), host(nk.split_lo(act)).view(np.uint32))


@pytest.mark.parametrize("B,T,H,D", [(2, 1024, 4, 64), (2, 300, 3, 64), (3, 200, 2, 32)])
def test_attn_with_given_lo_parts_bitwise(cuda, B, T, H, D):
    """ns_attn_fwd_lo / ns_attn_bwd_lo with qkv's lo part given equal the plain entries."""
    r = rng(B * T + H * D)
    C = H * D
    qkv = dev(normal(r, (B * T, 3 * C)), cuda)
    dout = dev(normal(r, (B * T, C)), cuda)
    qkv_lo = nk.split_lo(qkv)
    out, lse = nk.attn_fwd(qkv, B, T, H, D)
    out2, out_lo, lse2 = nk.attn_fwd_lo(qkv, qkv_lo, B, T, H, D)
    assert np.array_equal(host(out2).view(np.uint32), host(out).view(np.uint32))
    assert np.array_equal(host(lse2).view(np.uint32), host(lse).view(np.uint32))
    assert np.array_equal(host(out_lo).view(np.uint32), host(nk.split_lo(out)).view(np.uint32))
    want = nk.attn_bwd(qkv, out, dout, lse, B, T, H, D)
    got = nk.attn_bwd_lo(qkv, qkv_lo, out, dout, lse, B, T, H, D)
    assert np.array_equal(host(got).view(np.uint32), host(want).view(np.uint32))


def test_gelu_fwd_lo_matches_parts_bitwise(cuda):
    """ns_gelu_fwd_lo = ns_gelu_fwd + ns_split_lo, bit for bit (ragged length too)."""
    x = dev(normal(rng(34), (4 * 1024 * 1024 + 3,), std=2.0), cuda)
    y, lo = nk.gelu_fwd_lo(x)
    want = nk.gelu_fwd(x)
    assert np.array_equal(host(y).view(np.uint32), host(want).view(np.uint32))
    w = host(want)
    want_lo = w - (w.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
    assert np.array_equal(host(lo).view(np.uint32), want_lo.view(np.uint32))


@pytest.mark.parametrize("N,D", [(8192, 768), (300, 128), (257, 132), (64, 100), (77, 130)])
def test_layernorm_fwd_ex_matches_parts_bitwise(cuda, N, D):
    """ns_layernorm_fwd_ex = residual add (GEMM epilogue rounding) + LayerNorm + lo split.
    D=130 (not a multiple of 4) takes the scalar fallback path."""
    r = rng(N + D)
    raw = dev(normal(r, (N, D)), cuda)
    resid = dev(normal(r, (N, D)), cuda)
    bias = dev(normal(r, (D,)), cuda)
    gamma = dev(normal(r, (D,)), cuda)
    beta = dev(normal(r, (D,)), cuda)
    want_x = (host(raw) + host(bias)[None, :]).astype(np.float32) + host(resid)
    x, y, lo, mean, rstd = nk.layernorm_fwd_ex(raw, gamma, beta, bias=bias, resid=resid)
    assert np.array_equal(host(x).view(np.uint32), want_x.astype(np.float32).view(np.uint32))
    y2, m2, r2 = nk.layernorm_fwd(x, gamma, beta)
    for a, b in ((y, y2), (mean, m2), (rstd, r2)):
        assert np.array_equal(host(a).view(np.uint32), host(b).view(np.uint32))
    assert np.array_equal(host(lo).view(np.uint32), host(nk.split_lo(y2)).view(np.uint32))
    # plain LayerNorm with the lo output only
    _, y3, lo3, _, _ = nk.layernorm_fwd_ex(x, gamma, beta)
    assert np.array_equal(host(y3).view(np.uint32), host(y2).view(np.uint32))
    assert np.array_equal(host(lo3).view(np.uint32), host(lo).view(np.uint32))
    # the sum written over the GEMM product (x_out == x_raw), as GPTBlock does
    raw2 = raw.clone()
    x4, y4, lo4, _, _ = nk.layernorm_fwd_ex(raw2, gamma, beta, bias=bias, resid=resid,
                                            in_place=True)
    assert x4.data_ptr() == raw2.data_ptr()
    assert np.array_equal(host(x4).view(np.uint32), host(x).view(np.uint32))
    assert np.array_equal(host(y4).view(np.uint32), host(y).view(np.uint32))
    assert np.array_equal(host(lo4).view(np.uint32), host(lo).view(np.uint32))


def test_gemm_split_k_deterministic(cuda):
    """dW-shaped product that the planner splits over K: two runs, same bits."""
    M, Kd, N = 768, 8192, 768
    r = rng(9)
    X, dY = normal(r, (Kd, M)), normal(r, (Kd, N))
    Xd, dYd = dev(X, cuda), dev(dY, cuda)
    lib = _lib.load()
    assert lib.ns_gemm_workspace_size(M, N, Kd) > 0, "planner should split this shape"
    a = host(nk.gemm(Xd, dYd, a_trans=True))
    b = host(nk.gemm(Xd, dYd, a_trans=True))
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert rel_l2(a, fp64.matmul(X.T, dY)) < 1e-5
    c = host(nk.gemm(Xd, dYd, a_trans=True, split=False))
    assert rel_l2(c, fp64.matmul(X.T, dY)) < 1e-5


def test_gemm_rejects_bad_shapes(cuda):
    lib = _lib.load()
    rc = lib.ns_gemm(4, 4, 4, None, 2, 0, None, 4, 0, None, 4, 0.0, 0, None, None, None, None, 0, None)
    assert rc == _lib.NS_ERR_INVALID_ARGUMENT
    rc = lib.ns_gemm(4, 4, 4, None, 4, 0, None, 4, 0, None, 4, 0.5, 0, None, None, None, None, 0, None)
    assert rc == _lib.NS_ERR_INVALID_ARGUMENT


def test_bias_grad(cuda, port):
    for M, N in ((8192, 3072), (37, 19), (512, 384)):
        dY = normal(rng(M + N), (M, N))
        db = host(nk.bias_grad(dev(dY, cuda)))
        ref = np.zeros(N, np.float32)
        for i in range(M):
            ref += dY[i]
        assert_close(db, ref, fp64.f64(dY).sum(0), what=f"db {M}x{N}")


# -------------------------------------------------------------- attention

ATT_CASES = [(2, 64, 4, 32), (1, 8, 2, 8), (1, 1, 2, 4), (3, 16, 8, 4), (2, 5, 1, 4),
             (1, 32, 4, 16), (2, 100, 3, 64), (1, 70, 2, 128),
             # tensor-core shapes: T not a multiple of the 64-key / 128-query
             # blocks, one-token sequences, batches whose key blocks straddle
             # the next sequence
             (1, 1, 1, 64), (3, 33, 2, 32), (2, 129, 2, 64), (1, 300, 1, 64), (2, 200, 2, 32)]


@pytest.fixture(params=[0, 1], ids=["auto", "simt"])
def attn_engine(request):
    nk.attn_set_engine(request.param)
    yield request.param
    nk.attn_set_engine(0)


@pytest.mark.parametrize("B,T,H,D", ATT_CASES)
def test_attention_core(cuda, attn_engine, B, T, H, D):
    """Forward output and dqkv against the float64 restatement of the
    reference's per-(b,h) loop; includes the reference test_suite's
    fast-vs-literal shapes (test_suite.cpp:3112-3119).  Engine "auto" runs
    head sizes 32 and 64 on the tensor cores."""
    r = rng(B * 1000 + T * 10 + H + D)
    C = H * D
    qkv = normal(r, (B * T, 3 * C))
    dout = normal(r, (B * T, C))
    o64, p64 = fp64.attention_fwd(qkv, B, T, H, D)
    dq64 = fp64.attention_bwd(qkv, p64, dout, B, T, H, D)
    qd = dev(qkv, cuda)
    out, lse = nk.attn_fwd(qd, B, T, H, D)
    o = host(out)
    assert rel_l2(o, o64) < 1e-5
    assert np.allclose(o, o64, rtol=1e-4, atol=1e-5), np.abs(o - o64).max()
    # lse = m + log(sum exp(s - m)) per (b, h, row)
    q = qkv[:, :C].reshape(B, T, H, D).transpose(0, 2, 1, 3).astype(np.float64)
    k = qkv[:, C:2 * C].reshape(B, T, H, D).transpose(0, 2, 1, 3).astype(np.float64)
    s = q @ k.transpose(0, 1, 3, 2) / np.sqrt(D)
    s = np.where(np.tril(np.ones((T, T), bool)), s, -np.inf)
    mx = s.max(-1, keepdims=True)
    lse64 = (mx[..., 0] + np.log(np.exp(s - mx).sum(-1))).reshape(-1)
    assert np.allclose(host(lse), lse64, rtol=1e-5, atol=1e-5), np.abs(host(lse) - lse64).max()
    dq = host(nk.attn_bwd(qd, out, dev(dout, cuda), lse, B, T, H, D))
    assert rel_l2(dq, dq64) < 1e-5
    assert np.allclose(dq, dq64, rtol=1e-4, atol=1e-5), np.abs(dq - dq64).max()


@pytest.mark.parametrize("B,T,H,D", [(8, 1024, 12, 64), (2, 300, 3, 64), (3, 200, 2, 32),
                                     (1, 1, 1, 64), (2, 129, 2, 32)])
def test_attn_fused_dkdv_equals_separate_kernels_bitwise(cuda, B, T, H, D):
    """The fused dK+dV backward kernel (engine 0) performs the separate dV and
    dK kernels' operations in the same order (engine 2): same bits."""
    r = rng(B * T * H + D)
    C = H * D
    qkv = dev(normal(r, (B * T, 3 * C)), cuda)
    dout = dev(normal(r, (B * T, C)), cuda)
    out, lse = nk.attn_fwd(qkv, B, T, H, D)
    fused = host(nk.attn_bwd(qkv, out, dout, lse, B, T, H, D))
    nk.attn_set_engine(2)
    try:
        separate = host(nk.attn_bwd(qkv, out, dout, lse, B, T, H, D))
    finally:
        nk.attn_set_engine(0)
    assert np.array_equal(fused.view(np.uint32), separate.view(np.uint32))
    nk.kernel_health()


@pytest.mark.slow
def test_attention_full_size_deterministic(cuda):
    """B=8, T=1024, H=12, D=64: float64 check on two (b, h) slices, and two
    backward runs give identical bits (single-writer, no atomics)."""
    B, T, H, D = 8, 1024, 12, 64
    C = H * D
    r = rng(3)
    qkv = normal(r, (B * T, 3 * C))
    dout = normal(r, (B * T, C))
    qd, dd = dev(qkv, cuda), dev(dout, cuda)
    out, lse = nk.attn_fwd(qd, B, T, H, D)
    d1 = host(nk.attn_bwd(qd, out, dd, lse, B, T, H, D))
    d2 = host(nk.attn_bwd(qd, out, dd, lse, B, T, H, D))
    assert np.array_equal(d1.view(np.uint32), d2.view(np.uint32))
    # Check batch 5 in full (all heads) against float64.
    b = 5
    sl = slice(b * T, (b + 1) * T)
    o64, p64 = fp64.attention_fwd(qkv[sl], 1, T, H, D)
    dq64 = fp64.attention_bwd(qkv[sl], p64, dout[sl], 1, T, H, D)
    assert rel_l2(host(out)[sl], o64) < 1e-5
    assert rel_l2(d1[sl], dq64) < 1e-5


# ---------------------------------------------------- bandwidth kernels

@pytest.mark.parametrize("rows,dim", [(8192, 768), (512, 128), (13, 40), (7, 3), (33, 1030)])
def test_layernorm(cuda, port, rows, dim):
    r = rng(rows + dim)
    x = normal(r, (rows, dim), 2.0) + 0.5
    g = normal(r, dim) + 1.0
    b = normal(r, dim)
    dout = normal(r, (rows, dim))
    dres = normal(r, (rows, dim))
    o, m, s = nk.layernorm_fwd(dev(x, cuda), dev(g, cuda), dev(b, cuda))
    ro, rm, rs = port.layernorm_fwd(x, g, b)
    f_o, f_m, f_s = fp64.layernorm_fwd(x, g, b)
    assert_close(host(o), ro, f_o, what="ln out")
    assert_close(host(m), rm, f_m, what="ln mean")
    assert_close(host(s), rs, f_s, what="ln rstd")
    dx, dg, db = nk.layernorm_bwd(dev(dout, cuda), dev(x, cuda), dev(g, cuda), dev(rm, cuda),
                                 dev(rs, cuda), dresid=dev(dres, cuda))
    rdx, rdg, rdb = port.layernorm_bwd(dout, x, g, rm, rs)
    f_dx, f_dg, f_db = fp64.layernorm_bwd(dout, x, g, rm, rs)
    assert_close(host(dx), dres + rdx, dres + f_dx, what="ln dx+resid")
    assert_close(host(dg), rdg, f_dg, what="ln dgamma")
    assert_close(host(db), rdb, f_db, what="ln dbeta")


def test_layernorm_known_answer(cuda):
    """test_suite.cpp:120-133: mean of [2, 4, 4, 6] is 4."""
    x = dev(np.array([[2, 4, 4, 6]], np.float32), cuda)
    _, m, _ = nk.layernorm_fwd(x, dev(np.ones(4, np.float32), cuda), dev(np.zeros(4, np.float32), cuda))
    assert abs(float(host(m)[0]) - 4.0) < 1e-4


def test_gelu(cuda, port):
    x = normal(rng(2), 100003, 3.0)
    d = normal(rng(4), 100003)
    assert_close(host(nk.gelu_fwd(dev(x, cuda))), port.gelu_fwd(x), fp64.gelu(x), what="gelu")
    assert_close(host(nk.gelu_bwd(dev(d, cuda), dev(x, cuda))), port.gelu_bwd(d, x),
                 d * fp64.gelu_grad(x), what="gelu'")


def test_add_bit_exact(cuda):
    a, b = normal(rng(1), 1001), normal(rng(2), 1001)
    out = host(nk.add(dev(a, cuda), dev(b, cuda)))
    assert np.array_equal(out.view(np.uint32), (a + b).view(np.uint32))


@pytest.mark.parametrize("rows,V", [(8192, 256), (50, 256), (10, 11), (3, 1000)])
def test_cross_entropy(cuda, port, rows, V):
    r = rng(rows + V)
    logits = normal(r, (rows, V), 3.0)
    t = r.integers(0, V, rows)
    loss, d, err = nk.cross_entropy(dev(logits, cuda), dev(t, cuda, torch.int32))
    rl, rd = port.cross_entropy(logits, t.astype(np.float32))
    fl, fd = fp64.cross_entropy(logits, t)
    assert_close(host(loss), np.array([rl], np.float32), np.array([fl]), what="loss")
    assert_close(host(d), rd, fd, what="dlogits")
    assert int(host(err)[0]) == 0


def test_cross_entropy_bad_target_flag(cuda):
    logits = dev(normal(rng(1), (4, 8)), cuda)
    t = dev(np.array([0, 1, 8, 2]), cuda, torch.int32)
    _, _, err = nk.cross_entropy(logits, t)
    assert int(host(err)[0]) == 1


@pytest.mark.parametrize("B,T,V,C", [(8, 64, 256, 128), (2, 5, 11, 8), (8, 1024, 256, 768), (3, 7, 5, 6)])
def test_embedding_bit_exact(cuda, port, B, T, V, C):
    """Forward gather+add and the sorted-segment backward must reproduce the
    reference's sequential scatter-add bit for bit (embedding.h:61-80)."""
    r = rng(B + T + V + C)
    wte, wpe = normal(r, (V, C), 0.02), normal(r, (T + 3, C), 0.02)
    tok = r.integers(0, V, (B, T))
    tok[0, :] = tok[0, 0]  # long segment
    dx = normal(r, (B, T, C))
    head = normal(r, (V, C), 1e-3)
    x, err = nk.embedding_fwd(dev(tok, cuda, torch.int32), dev(wte, cuda), dev(wpe, cuda))
    ref_tok, _ = port.embedding(wte, tok.astype(np.float32))
    ref = ref_tok + wpe[:T][None]
    assert np.array_equal(host(x).view(np.uint32), ref.view(np.uint32))
    assert int(host(err)[0]) == 0
    dwte_d = dev(head, cuda)
    dwte, dwpe = nk.embedding_bwd(dev(tok, cuda, torch.int32), dev(dx, cuda), V, T + 3,
                                 dwte=dwte_d, accumulate_wte=True)
    _, ref_dw = port.embedding(wte, tok.astype(np.float32), dx)
    want = ref_dw + head  # gpt.h:266-269: embedding sum first, then += head term
    assert np.array_equal(host(dwte).view(np.uint32), want.view(np.uint32))
    want_pe = np.zeros((T + 3, C), np.float32)
    for b in range(B):
        want_pe[:T] += dx[b]
    assert np.array_equal(host(dwpe).view(np.uint32), want_pe.view(np.uint32))


def test_embedding_out_of_range(cuda):
    wte, wpe = dev(np.zeros((10, 4), np.float32), cuda), dev(np.zeros((2, 4), np.float32), cuda)
    _, err = nk.embedding_fwd(dev(np.array([[0, 999]]), cuda, torch.int32), wte, wpe)
    assert int(host(err)[0]) == 1
    with pytest.raises(IndexError):
        nk.embedding_fwd(dev(np.zeros((1, 3)), cuda, torch.int32), wte, wpe)  # T > block


def test_adamw_bit_exact(cuda, port):
    """ns_adamw_flat against the oracle's AdamW::Step on the same gradients,
    three steps, rank>=2 tensors decayed (optimizers.h:206-234)."""
    r = rng(8)
    sizes = [1000, 7, 130, 4096 * 33 + 5, 3]
    decay = [0.01, 0.0, 0.01, 0.01, 0.0]
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    n = int(offs[-1])
    p = normal(r, n, 0.02)
    p_ref, m_ref, v_ref = p.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    pd = dev(p, cuda)
    md = torch.zeros(n, device=cuda)
    vd = torch.zeros(n, device=cuda)
    lr, b1, b2, eps = 3e-4, 0.9, 0.95, 1e-8
    for step in (1, 2, 3):
        g = normal(r, n, 0.1)
        port.adamw_flat(p_ref, g, m_ref, v_ref, offs, decay, lr, b1, b2, eps, step)
        bc1 = np.float32(1.0 - np.power(np.float64(np.float32(b1)), step))
        bc2 = np.float32(1.0 - np.power(np.float64(np.float32(b2)), step))
        nk.adamw_flat(pd, dev(g, cuda), md, vd, offs.tolist(), decay, lr, b1, b2, eps, float(bc1),
                     float(bc2))
    assert np.array_equal(host(pd).view(np.uint32), p_ref.view(np.uint32))
    assert np.array_equal(host(md).view(np.uint32), m_ref.view(np.uint32))
    assert np.array_equal(host(vd).view(np.uint32), v_ref.view(np.uint32))


def test_adamw_many_tensors_bit_exact(cuda, port):
    """More tensors than one launch's segment table holds (two launches), empty
    tensors, odd sizes and CTA shares that cross tensor boundaries, against the
    oracle's AdamW::Step bit for bit."""
    r = rng(9)
    sizes = [int(x) for x in r.integers(0, 300, 700)]
    sizes[5] = sizes[6] = 0
    sizes[400] = 250_003
    decay = [0.01 if i % 3 else 0.0 for i in range(len(sizes))]
    offs = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
    n = int(offs[-1])
    p = normal(r, n, 0.02)
    p_ref, m_ref, v_ref = p.copy(), np.zeros(n, np.float32), np.zeros(n, np.float32)
    pd, md, vd = dev(p, cuda), torch.zeros(n, device=cuda), torch.zeros(n, device=cuda)
    lr, b1, b2, eps = 1e-3, 0.9, 0.95, 1e-8
    for step in (1, 2):
        g = normal(r, n, 0.1)
        port.adamw_flat(p_ref, g, m_ref, v_ref, offs, decay, lr, b1, b2, eps, step)
        bc1 = np.float32(1.0 - np.power(np.float64(np.float32(b1)), step))
        bc2 = np.float32(1.0 - np.power(np.float64(np.float32(b2)), step))
        nk.adamw_flat(pd, dev(g, cuda), md, vd, offs.tolist(), decay, lr, b1, b2, eps, float(bc1),
                      float(bc2))
    assert np.array_equal(host(pd).view(np.uint32), p_ref.view(np.uint32))
    assert np.array_equal(host(md).view(np.uint32), m_ref.view(np.uint32))
    assert np.array_equal(host(vd).view(np.uint32), v_ref.view(np.uint32))


def test_sumsq_and_clip(cuda):
    x = normal(rng(3), 100001, 0.1)
    s = nk.sumsq(dev(x, cuda))
    assert abs(float(host(s)[0]) - float((x.astype(np.float64) ** 2).sum())) < 1e-4 * float((x.astype(np.float64) ** 2).sum())
    xd = dev(x, cuda)
    nk.clip_scale(xd, s, 1.0)
    norm = np.sqrt((x.astype(np.float64) ** 2).sum())
    assert np.allclose(host(xd), x * (1.0 / norm), rtol=1e-5, atol=1e-8)
