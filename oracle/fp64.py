"""Test infrastructure: float64 numpy restatement of the GPT training step. NOT product code.

Used in two ways by the tests:

* as the adjudicator of float tolerances (the approach of the reference's
  tools/parity/precision_probe.py:91-96): where the CUDA result and the fp32
  reference differ by more than the stated tolerance, the element passes only
  if the CUDA result is no farther from this float64 computation than the fp32
  reference is;
* as the checker at sizes where the fp32 C oracle would take minutes (the
  MatMul sweep at 8192-16384 rows, attention at T=1024).

Each function states the reference function it restates (paths inside the
NeuralSuite project).  Layouts are the reference's (row-major).
"""
from __future__ import annotations

import numpy as np

GELU_C = 0.7978845608
GELU_A = 0.044715


def f64(a):
    return np.asarray(a, dtype=np.float64)


def matmul(A, B):
    """src/tensor.cpp:198-271 (exact product, float64 accumulation)."""
    return f64(A) @ f64(B)


def gelu(x):
    """src/tensor.cpp:428-443"""
    x = f64(x)
    return 0.5 * x * (1.0 + np.tanh(GELU_C * (x + GELU_A * x ** 3)))


def gelu_grad(x):
    """src/tensor.cpp:445-461 (the derivative factor)."""
    x = f64(x)
    th = np.tanh(GELU_C * (x + GELU_A * x ** 3))
    return 0.5 * (1.0 + th) + 0.5 * x * (1.0 - th * th) * GELU_C * (1.0 + 3.0 * GELU_A * x * x)


def layernorm_fwd(x, g, b, eps=1e-5):
    """src/tensor.cpp:290-322"""
    x = f64(x)
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    rs = 1.0 / np.sqrt(v + eps)
    return (x - m) * rs * f64(g) + f64(b), m[..., 0], rs[..., 0]


def layernorm_bwd(dout, x, g, mean, rstd):
    """src/tensor.cpp:324-359"""
    x, dout, g = f64(x), f64(dout), f64(g)
    D = x.shape[-1]
    xh = (x - f64(mean)[..., None]) * f64(rstd)[..., None]
    dxh = dout * g
    s1 = dxh.sum(-1, keepdims=True)
    s2 = (dxh * xh).sum(-1, keepdims=True)
    dx = (f64(rstd)[..., None] / D) * (D * dxh - s1 - xh * s2)
    rows = dout.reshape(-1, D)
    return dx, (rows * xh.reshape(-1, D)).sum(0), rows.sum(0)


def cross_entropy(logits, targets):
    """include/losses.h:34-86 -> (mean loss, dlogits)."""
    z = f64(logits)
    t = np.asarray(targets).astype(np.int64)
    z = z - z.max(-1, keepdims=True)
    lse = np.log(np.exp(z).sum(-1))
    n = z.shape[0]
    loss = float(np.mean(lse - z[np.arange(n), t]))
    p = np.exp(z - lse[:, None])
    p[np.arange(n), t] -= 1.0
    return loss, p / n


def attention_fwd(qkv, B, T, H, D):
    """Core of MultiHeadAttention::Forward (include/layers/attention.h:364-384).

    Returns out [B*T, C] and the probabilities [B, H, T, T]."""
    C = H * D
    x = f64(qkv).reshape(B, T, 3, H, D)
    q = x[:, :, 0].transpose(0, 2, 1, 3)
    k = x[:, :, 1].transpose(0, 2, 1, 3)
    v = x[:, :, 2].transpose(0, 2, 1, 3)
    s = (q @ k.transpose(0, 1, 3, 2)) * (1.0 / np.sqrt(D))
    mask = np.triu(np.ones((T, T), dtype=bool), 1)
    s = np.where(mask, -np.inf, s)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    o = p @ v
    return o.transpose(0, 2, 1, 3).reshape(B * T, C), p


def attention_bwd(qkv, p, dout, B, T, H, D):
    """Core of MultiHeadAttention::Backward (include/layers/attention.h:405-461)."""
    C = H * D
    x = f64(qkv).reshape(B, T, 3, H, D)
    q = x[:, :, 0].transpose(0, 2, 1, 3)
    k = x[:, :, 1].transpose(0, 2, 1, 3)
    v = x[:, :, 2].transpose(0, 2, 1, 3)
    do = f64(dout).reshape(B, T, H, D).transpose(0, 2, 1, 3)
    scale = 1.0 / np.sqrt(D)
    dp = do @ v.transpose(0, 1, 3, 2)
    dv = p.transpose(0, 1, 3, 2) @ do
    ds = p * (dp - (dp * p).sum(-1, keepdims=True)) * scale
    dq = ds @ k
    dk = ds.transpose(0, 1, 3, 2) @ q
    out = np.zeros((B, T, 3, H, D))
    out[:, :, 0] = dq.transpose(0, 2, 1, 3)
    out[:, :, 1] = dk.transpose(0, 2, 1, 3)
    out[:, :, 2] = dv.transpose(0, 2, 1, 3)
    return out.reshape(B * T, 3 * C)


def param_shapes(V, block, L, C):
    """Registration order of GPTModel::Parameters() (include/gpt.h:143-149, 59-63)."""
    shapes = [(V, C), (block, C)]
    for _ in range(L):
        shapes += [(C,), (C,), (C, 3 * C), (3 * C,), (C, C), (C,), (C,), (C,), (C, 4 * C),
                   (4 * C,), (4 * C, C), (C,)]
    shapes += [(C,), (C,)]
    return shapes


def split_params(flat, V, block, L, C):
    out, off = [], 0
    for s in param_shapes(V, block, L, C):
        n = int(np.prod(s))
        out.append(f64(flat[off:off + n]).reshape(s))
        off += n
    return out


def gpt_fwd_bwd(flat, idx, targets, V, block, L, H, C, keep_probs=True):
    """GPTModel Forward -> CrossEntropy -> Backward (include/gpt.h:192-272) in float64.

    keep_probs=False recomputes each layer's [B,H,T,T] probabilities in the
    backward instead of keeping all of them (9.7 GB at 12 layers, B=8,
    T=1024, H=12), the same numbers with less memory.
    Returns (loss, logits [B,T,V], grads flat)."""
    P = split_params(flat, V, block, L, C)
    idx = np.asarray(idx).astype(np.int64)
    B, T = idx.shape
    M, D = B * T, C // H
    wte, wpe = P[0], P[1]
    x = (wte[idx] + wpe[np.arange(T)][None]).reshape(M, C)
    caches = []
    for l in range(L):
        g1, b1, Wa, ba, Wp, bp, g2, b2, Wf, bf, Wm, bm = P[2 + 12 * l: 14 + 12 * l]
        h1, m1, r1 = layernorm_fwd(x, g1, b1)
        qkv = h1 @ Wa + ba
        att, probs = attention_fwd(qkv, B, T, H, D)
        if not keep_probs:
            probs = None
        x1 = x + (att @ Wp + bp)
        h2, m2, r2 = layernorm_fwd(x1, g2, b2)
        fc = h2 @ Wf + bf
        ge = gelu(fc)
        x2 = x1 + (ge @ Wm + bm)
        caches.append((x, h1, m1, r1, qkv, att, probs, x1, h2, m2, r2, fc, ge))
        x = x2
    gf, bfn = P[-2], P[-1]
    xf, mf, rf = layernorm_fwd(x, gf, bfn)
    logits = xf @ wte.T
    loss, dl = cross_entropy(logits, np.asarray(targets).reshape(-1))
    G = [np.zeros_like(p) for p in P]
    dx = dl @ wte
    dwte_head = dl.T @ xf
    dcur, G[-2], G[-1] = layernorm_bwd(dx, x, gf, mf, rf)
    for l in reversed(range(L)):
        g1, b1, Wa, ba, Wp, bp, g2, b2, Wf, bf, Wm, bm = P[2 + 12 * l: 14 + 12 * l]
        xin, h1, m1, r1, qkv, att, probs, x1, h2, m2, r2, fc, ge = caches[l]
        o = 2 + 12 * l
        G[o + 10] = ge.T @ dcur
        G[o + 11] = dcur.sum(0)
        dge = (dcur @ Wm.T) * gelu_grad(fc)
        G[o + 8] = h2.T @ dge
        G[o + 9] = dge.sum(0)
        dh2 = dge @ Wf.T
        dxn2, G[o + 6], G[o + 7] = layernorm_bwd(dh2, x1, g2, m2, r2)
        dx1 = dcur + dxn2
        G[o + 4] = att.T @ dx1
        G[o + 5] = dx1.sum(0)
        datt = dx1 @ Wp.T
        if probs is None:
            probs = attention_fwd(qkv, B, T, H, D)[1]
        dqkv = attention_bwd(qkv, probs, datt, B, T, H, D)
        del probs
        G[o + 2] = h1.T @ dqkv
        G[o + 3] = dqkv.sum(0)
        dh1 = dqkv @ Wa.T
        dxn1, G[o + 0], G[o + 1] = layernorm_bwd(dh1, xin, g1, m1, r1)
        dcur = dx1 + dxn1
    dwte = np.zeros_like(wte)
    np.add.at(dwte, idx.reshape(-1), dcur)
    G[0] = dwte + dwte_head
    dwpe = np.zeros_like(wpe)
    dwpe[:T] = dcur.reshape(B, T, C).sum(0)
    G[1] = dwpe
    return loss, logits.reshape(B, T, V), np.concatenate([g.reshape(-1) for g in G])


def gpt_decode(flat, steps, V, block, L, H, C):
    """GPTModel::ForwardWithKVCache (include/gpt.h:159-190) in float64 for one
    sequence: steps is a list of (token, pos); each step appends its K and V
    to the cache (include/layers/attention.h:481-546) and returns the
    logits [V] of that step.  Returns an array [len(steps), V]."""
    P = split_params(flat, V, block, L, C)
    D = C // H
    wte, wpe = P[0], P[1]
    kc = [[] for _ in range(L)]
    vc = [[] for _ in range(L)]
    out = []
    for tok, pos in steps:
        x = wte[int(tok)] + wpe[int(pos)]
        for l in range(L):
            g1, b1, Wa, ba, Wp, bp, g2, b2, Wf, bf, Wm, bm = P[2 + 12 * l: 14 + 12 * l]
            h1 = layernorm_fwd(x[None], g1, b1)[0][0]
            qkv = h1 @ Wa + ba
            q = qkv[:C].reshape(H, D)
            kc[l].append(qkv[C:2 * C].reshape(H, D))
            vc[l].append(qkv[2 * C:].reshape(H, D))
            K = np.stack(kc[l], 1)  # [H, t, D]
            Vv = np.stack(vc[l], 1)
            s = np.einsum("hd,htd->ht", q, K) / np.sqrt(D)
            s = np.exp(s - s.max(-1, keepdims=True))
            p = s / s.sum(-1, keepdims=True)
            att = np.einsum("ht,htd->hd", p, Vv).reshape(C)
            x1 = x + (att @ Wp + bp)
            h2 = layernorm_fwd(x1[None], g2, b2)[0][0]
            x = x1 + (gelu(h2 @ Wf + bf) @ Wm + bm)
        xf = layernorm_fwd(x[None], P[-2], P[-1])[0][0]
        out.append(xf @ wte.T)
    return np.array(out)


def _im2col(x, k, s, p):
    """[B, IC, H, W] -> columns [B, IC*k*k, OH*OW] (Conv2D's Im2Col,
    include/layers/conv2d.h:348-375), float64."""
    x = f64(x)
    B, IC, H, W = x.shape
    OH, OW = (H + 2 * p - k) // s + 1, (W + 2 * p - k) // s + 1
    xp = np.zeros((B, IC, H + 2 * p, W + 2 * p))
    xp[:, :, p:p + H, p:p + W] = x
    cols = np.empty((B, IC, k, k, OH, OW))
    for kh in range(k):
        for kw in range(k):
            cols[:, :, kh, kw] = xp[:, :, kh:kh + s * OH:s, kw:kw + s * OW:s]
    return cols.reshape(B, IC * k * k, OH * OW), OH, OW


def conv2d_fwd(x, w, b, s, p):
    """Conv2D::Forward (include/layers/conv2d.h:211-266) in float64."""
    OC, IC, k, _ = w.shape
    cols, OH, OW = _im2col(x, k, s, p)
    y = np.einsum("ok,bkp->bop", f64(w).reshape(OC, -1), cols) + f64(b)[None, :, None]
    return y.reshape(x.shape[0], OC, OH, OW)


def conv2d_bwd(x, w, dy, s, p):
    """Conv2D::Backward (include/layers/conv2d.h:268-331) in float64 -> (dx, dw, db)."""
    OC, IC, k, _ = w.shape
    B, _, H, W = x.shape
    cols, OH, OW = _im2col(x, k, s, p)
    d = f64(dy).reshape(B, OC, OH * OW)
    dw = np.einsum("bop,bkp->ok", d, cols).reshape(w.shape)
    db = d.sum((0, 2))
    dcols = np.einsum("ok,bop->bkp", f64(w).reshape(OC, -1), d).reshape(B, IC, k, k, OH, OW)
    dxp = np.zeros((B, IC, H + 2 * p, W + 2 * p))
    for kh in range(k):
        for kw in range(k):
            dxp[:, :, kh:kh + s * OH:s, kw:kw + s * OW:s] += dcols[:, :, kh, kw]
    return dxp[:, :, p:p + H, p:p + W], dw, db


def unet_fwd_bwd(flat, sizes, x, target, in_ch, base, hw):
    """The diffusion U-Net step of ref_harness.cpp in float64: forward, MSE,
    backward.  sizes: the tensor sizes in registration order.  Returns
    (loss, prediction, grads flat).  Nearest 2x upsampling is the only layer
    the reference does not have."""
    parts, off = [], 0
    for n in sizes:
        parts.append(f64(flat[off:off + n]))
        off += n
    c = [base, 2 * base, 4 * base, 2 * base, base]
    w = [hw, hw // 2, hw // 4, hw // 2, hw]
    cin = [in_ch, base, 2 * base, 4 * base, 2 * base]
    stride = [1, 2, 2, 1, 1]
    # per level: conv (w, b), res conv (w, b), ln (g, b); then conv_out (w, b)
    P = []
    for l in range(5):
        k = 6 * l
        P.append(dict(cw=parts[k].reshape(c[l], cin[l], 3, 3), cb=parts[k + 1],
                      rw=parts[k + 2].reshape(c[l], c[l], 3, 3), rb=parts[k + 3],
                      g=parts[k + 4], b=parts[k + 5]))
    ow, ob = parts[30].reshape(in_ch, base, 3, 3), parts[31]

    def up(t):
        return t.repeat(2, axis=2).repeat(2, axis=3)

    def up_bwd(d):
        B, C, H, W = d.shape
        return d.reshape(B, C, H // 2, 2, W // 2, 2).sum((3, 5))

    cache = []

    def level_fwd(l, inp, skip=None):
        a = conv2d_fwd(inp, P[l]["cw"], P[l]["cb"], stride[l], 1)
        if skip is not None:
            a = a + skip
        f = conv2d_fwd(a, P[l]["rw"], P[l]["rb"], 1, 1)
        r = np.maximum(f + a, 0.0)
        e, m, s = layernorm_fwd(r, P[l]["g"], P[l]["b"])
        cache.append((inp, a, r, m, s))
        return e

    x = f64(x)
    e0 = level_fwd(0, x)
    e1 = level_fwd(1, e0)
    mm = level_fwd(2, e1)
    u1 = level_fwd(3, up(mm), e1)
    u0 = level_fwd(4, up(u1), e0)
    y = conv2d_fwd(u0, ow, ob, 1, 1)
    n = y.size
    diff = y - f64(target)
    loss = float((diff * diff).sum() / n)
    dy = 2.0 * diff / n
    G = [None] * 32

    def level_bwd(l, de):
        inp, a, r, m, s = cache[l]
        dr, G[6 * l + 4], G[6 * l + 5] = layernorm_bwd(de, r, P[l]["g"], m, s)
        dsum = np.where(r > 0, dr, 0.0)
        dfa, G[6 * l + 2], G[6 * l + 3] = conv2d_bwd(a, P[l]["rw"], dsum, 1, 1)
        da = dfa + dsum
        dinp, G[6 * l], G[6 * l + 1] = conv2d_bwd(inp, P[l]["cw"], da, stride[l], 1)
        return dinp, da

    du0, G[30], G[31] = conv2d_bwd(u0, ow, dy, 1, 1)
    dup1, ds0 = level_bwd(4, du0)
    dup0, ds1 = level_bwd(3, up_bwd(dup1))
    de1_part, _ = level_bwd(2, up_bwd(dup0))
    de0_part, _ = level_bwd(1, de1_part + ds1)
    level_bwd(0, de0_part + ds0)
    return loss, y, np.concatenate([g.reshape(-1) for g in G])


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def lstm_fwd_bwd(x, w_ih, w_hh, b_ih, b_hh, dout):
    """LSTM::Forward / ::Backward (include/layers/lstm.h:348-529) in float64:
    returns (out [T,B,H], dx, [dW_ih, dW_hh, db_ih, db_hh])."""
    x, w_ih, w_hh, b = f64(x), f64(w_ih), f64(w_hh), f64(b_ih) + f64(b_hh)
    T, B, _ = x.shape
    H = w_hh.shape[1]
    h = np.zeros((B, H))
    c = np.zeros((B, H))
    cache, outs = [], []
    for t in range(T):
        pre = x[t] @ w_ih.T + h @ w_hh.T + b
        i, f, g, o = (_sigmoid(pre[:, :H]), _sigmoid(pre[:, H:2 * H]), np.tanh(pre[:, 2 * H:3 * H]),
                      _sigmoid(pre[:, 3 * H:]))
        c_new = f * c + i * g
        tc = np.tanh(c_new)
        cache.append((h, c, i, f, g, o, tc))
        h, c = o * tc, c_new
        outs.append(h)
    d = f64(dout)
    dW_ih, dW_hh, db = np.zeros_like(w_ih), np.zeros_like(w_hh), np.zeros(4 * H)
    dx = np.zeros_like(x)
    dh_next = np.zeros((B, H))
    dc_next = np.zeros((B, H))
    for t in reversed(range(T)):
        h_prev, c_prev, i, f, g, o, tc = cache[t]
        dh = d[t] + dh_next
        dc = dh * o * (1 - tc * tc) + dc_next
        dpre = np.concatenate([dc * g * i * (1 - i), dc * c_prev * f * (1 - f),
                               dc * i * (1 - g * g), dh * tc * o * (1 - o)], 1)
        dc_next = dc * f
        dh_next = dpre @ w_hh
        dW_ih += dpre.T @ x[t]
        dW_hh += dpre.T @ h_prev
        db += dpre.sum(0)
        dx[t] = dpre @ w_ih
    return np.stack(outs), dx, [dW_ih, dW_hh, db, db.copy()]


def bilstm_fwd_bwd(x, wf, wr, dout):
    """BiLSTM (include/layers/lstm.h:531-664) in float64; wf / wr are
    (w_ih, w_hh, b_ih, b_hh).  Returns (out [T,B,2H], dx, grads fwd + rev)."""
    H = f64(wf[1]).shape[1]
    d = f64(dout)
    of, dxf, gf = lstm_fwd_bwd(x, *wf, d[:, :, :H])
    orr, dxr, gr = lstm_fwd_bwd(f64(x)[::-1], *wr, d[::-1, :, H:])
    return np.concatenate([of, orr[::-1]], 2), dxf + dxr[::-1], gf + gr
