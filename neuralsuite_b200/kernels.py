"""Tensor-level wrappers of the kernel entry points of the C ABI.

Each function takes CUDA torch tensors (fp32, contiguous; int32 for token ids),
calls exactly one ``ns_*`` entry point on the current torch stream and returns
the outputs.  Torch is only the allocator here; every number is produced by
libns_b200.so.  The reference function each wrapper stands for is named in its
docstring (paths inside the NeuralSuite project).
"""
from __future__ import annotations

import torch

from . import _lib

_f32 = torch.float32


def _p(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _req(t, name, dtype=_f32):
    if not (t.is_cuda and t.dtype == dtype and t.is_contiguous()):
        raise ValueError(f"{name} must be a contiguous CUDA {dtype} tensor")


def _ws(nbytes, device):
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def set_gemm_engine(engine: int) -> None:
    """0 = automatic (tcgen05 where TMA allows), 1 = SIMT fp32 everywhere,
    2 = tcgen05 with the operand split done inside the kernel, 3 / 4 = only
    256 x 256 CTA-pair / 128 x 256 tiles (pre-split operands), 5 = as 4 with
    row stores, 6 / 7 / 8 = pair tiles 256 x 192 / 256 x 128 / 256 x 256 only,
    9 = automatic without the stream-K tail, 10 / 11 = automatic with the
    CTA-pair kernel's work always handed out in a fixed order / always from a
    per-launch counter (engine 0: fixed, except in a data-parallel GPT
    backward; bit-identical results).  Engines 1-11 are for tests
    and profiling."""
    _lib.check(_lib.load().ns_gemm_set_engine(engine))


def kernel_health() -> None:
    _lib.check(_lib.load().ns_kernel_health())


def split_lo(x):
    """tf32 lo part of a 2-D fp32 tensor (x - trunc_tf32(x)), compact."""
    lib = _lib.load()
    _req(x, "x")
    lo = torch.empty_like(x)
    _lib.check(lib.ns_split_lo(_p(x), x.shape[0], x.shape[1], x.shape[1], _p(lo), _stream()))
    return lo


def gemm(A, B, a_trans=False, b_trans=False, epilogue=_lib.EPI_STORE, bias=None, aux=None,
         out=None, aux_out=None, beta=0.0, split=True, a_lo=None, b_lo=None, out_lo=None):
    """MatMul (src/tensor.cpp:198-271) with transposed operands read in place.

    ``A`` is [M,K] (or [K,M] if a_trans), ``B`` is [K,N] (or [N,K] if b_trans).
    ``a_lo`` / ``b_lo``: lo parts from split_lo of the same tensors (ns_gemm_lo).
    ``out_lo``: receives the tf32 lo part of the activation output (ns_gemm_lo_out).
    """
    lib = _lib.load()
    _req(A, "A")
    _req(B, "B")
    M, K = (A.shape[1], A.shape[0]) if a_trans else (A.shape[0], A.shape[1])
    KB, N = (B.shape[1], B.shape[0]) if b_trans else (B.shape[0], B.shape[1])
    if K != KB:
        raise ValueError(f"gemm: inner dimensions differ ({K} vs {KB})")
    if out is None:
        out = torch.empty((M, N), dtype=_f32, device=A.device)
    if epilogue == _lib.EPI_BIAS_GELU and aux_out is None:
        aux_out = torch.empty((M, N), dtype=_f32, device=A.device)
    ws_bytes = lib.ns_gemm_workspace_size(M, N, K) if split else 0
    ws = _ws(ws_bytes, A.device) if ws_bytes else None
    if out_lo is not None:
        _lib.check(lib.ns_gemm_lo_out(M, N, K, _p(A), A.shape[1], int(a_trans), _p(a_lo), _p(B),
                                      B.shape[1], int(b_trans), _p(b_lo), _p(out), out.shape[1],
                                      float(beta), epilogue, _p(bias), _p(aux), _p(aux_out),
                                      _p(out_lo), _p(ws), ws_bytes, _stream()))
    elif a_lo is None and b_lo is None:
        _lib.check(lib.ns_gemm(M, N, K, _p(A), A.shape[1], int(a_trans), _p(B), B.shape[1],
                               int(b_trans), _p(out), out.shape[1], float(beta), epilogue,
                               _p(bias), _p(aux), _p(aux_out), _p(ws), ws_bytes, _stream()))
    else:
        _lib.check(lib.ns_gemm_lo(M, N, K, _p(A), A.shape[1], int(a_trans), _p(a_lo), _p(B),
                                  B.shape[1], int(b_trans), _p(b_lo), _p(out), out.shape[1],
                                  float(beta), epilogue, _p(bias), _p(aux), _p(aux_out), _p(ws),
                                  ws_bytes, _stream()))
    return (out, aux_out) if epilogue == _lib.EPI_BIAS_GELU else out


def bias_grad(dY):
    """db = column sums of dY (include/layers/linear.h:104-111)."""
    lib = _lib.load()
    _req(dY, "dY")
    M, N = dY.shape
    db = torch.empty(N, dtype=_f32, device=dY.device)
    nb = lib.ns_bias_grad_workspace_size(M, N)
    ws = _ws(nb, dY.device)
    _lib.check(lib.ns_bias_grad(_p(dY), M, N, _p(db), _p(ws), nb, _stream()))
    return db


def attn_fwd(qkv, B, T, H, D):
    """MultiHeadAttention core forward (include/layers/attention.h:364-384)."""
    lib = _lib.load()
    _req(qkv, "qkv")
    out = torch.empty((B * T, H * D), dtype=_f32, device=qkv.device)
    lse = torch.empty((B * H * T,), dtype=_f32, device=qkv.device)
    nb = lib.ns_attn_fwd_workspace_size(B, T, H, D)
    ws = _ws(nb, qkv.device)
    _lib.check(lib.ns_attn_fwd(_p(qkv), B, T, H, D, _p(out), _p(lse), _p(ws), nb, _stream()))
    return out, lse


def attn_fwd_lo(qkv, qkv_lo, B, T, H, D):
    """(out, out_lo, lse) with qkv's lo part given (ns_attn_fwd_lo)."""
    lib = _lib.load()
    _req(qkv, "qkv")
    out = torch.empty((B * T, H * D), dtype=_f32, device=qkv.device)
    out_lo = torch.empty_like(out)
    lse = torch.empty((B * H * T,), dtype=_f32, device=qkv.device)
    nb = 0 if qkv_lo is not None else lib.ns_attn_fwd_workspace_size(B, T, H, D)
    ws = _ws(nb, qkv.device) if nb else None
    _lib.check(lib.ns_attn_fwd_lo(_p(qkv), _p(qkv_lo), B, T, H, D, _p(out), _p(out_lo), _p(lse),
                                  _p(ws), nb, _stream()))
    return out, out_lo, lse


def attn_bwd_lo(qkv, qkv_lo, out, dout, lse, B, T, H, D):
    """ns_attn_bwd with qkv's lo part given (ns_attn_bwd_lo)."""
    lib = _lib.load()
    dqkv = torch.empty_like(qkv)
    nb = lib.ns_attn_bwd_workspace_size(B, T, H, D)
    ws = _ws(nb, qkv.device)
    _lib.check(lib.ns_attn_bwd_lo(_p(qkv), _p(qkv_lo), _p(out), _p(dout), _p(lse), B, T, H, D,
                                  _p(dqkv), _p(ws), nb, _stream()))
    return dqkv


def attn_set_engine(engine):
    """0: tensor-core attention where the head size has a kernel (dK and dV
    from one backward kernel); 1: SIMT only; 2: as 0 with dK and dV from two
    kernels."""
    _lib.check(_lib.load().ns_attn_set_engine(engine))


def attn_bwd(qkv, out, dout, lse, B, T, H, D):
    """MultiHeadAttention core backward (include/layers/attention.h:405-461)."""
    lib = _lib.load()
    for t, n in ((qkv, "qkv"), (out, "out"), (dout, "dout"), (lse, "lse")):
        _req(t, n)
    dqkv = torch.empty_like(qkv)
    nb = lib.ns_attn_bwd_workspace_size(B, T, H, D)
    ws = _ws(nb, qkv.device)
    _lib.check(lib.ns_attn_bwd(_p(qkv), _p(out), _p(dout), _p(lse), B, T, H, D, _p(dqkv), _p(ws),
                               nb, _stream()))
    return dqkv


def bias_grad_split(dY):
    """(db, lo part of dY) from one pass (ns_bias_grad_split)."""
    lib = _lib.load()
    _req(dY, "dY")
    M, N = dY.shape
    db = torch.empty(N, dtype=_f32, device=dY.device)
    lo = torch.empty_like(dY)
    nb = lib.ns_bias_grad_workspace_size(M, N)
    ws = _ws(nb, dY.device)
    _lib.check(lib.ns_bias_grad_split(_p(dY), M, N, _p(db), _p(lo), _p(ws), nb, _stream()))
    return db, lo


def bias_grad_split_gelu(dY, pre):
    """dY * gelu'(pre) (in place), its column sums and its lo part (ns_bias_grad_split_gelu)."""
    lib = _lib.load()
    _req(dY, "dY")
    _req(pre, "pre")
    M, N = dY.shape
    db = torch.empty(N, dtype=_f32, device=dY.device)
    lo = torch.empty_like(dY)
    nb = lib.ns_bias_grad_workspace_size(M, N)
    ws = _ws(nb, dY.device)
    _lib.check(lib.ns_bias_grad_split_gelu(_p(dY), _p(pre), M, N, _p(db), _p(lo), _p(ws), nb,
                                           _stream()))
    return dY, db, lo


def layernorm_fwd(x, gamma, beta, eps=1e-5):
    """LayerNormForward (src/tensor.cpp:290-322)."""
    lib = _lib.load()
    _req(x, "x")
    D = x.shape[-1]
    N = x.numel() // D
    out = torch.empty_like(x)
    mean = torch.empty(N, dtype=_f32, device=x.device)
    rstd = torch.empty(N, dtype=_f32, device=x.device)
    _lib.check(lib.ns_layernorm_fwd(_p(x), _p(gamma), _p(beta), _p(out), _p(mean), _p(rstd), N, D,
                                    eps, _stream()))
    return out, mean, rstd


def layernorm_fwd_ex(raw, gamma, beta, bias=None, resid=None, want_lo=True, eps=1e-5,
                     in_place=False):
    """ns_layernorm_fwd_ex: (x, y, y_lo, mean, rstd) with x = resid + (raw + bias) if resid
    given; in_place writes x over raw (as the model does)."""
    lib = _lib.load()
    D = raw.shape[-1]
    N = raw.numel() // D
    x = (raw if in_place else torch.empty_like(raw)) if resid is not None else None
    y = torch.empty_like(raw)
    lo = torch.empty_like(raw) if want_lo else None
    mean = torch.empty(N, dtype=_f32, device=raw.device)
    rstd = torch.empty(N, dtype=_f32, device=raw.device)
    _lib.check(lib.ns_layernorm_fwd_ex(_p(raw), _p(bias), _p(resid), _p(x), _p(gamma), _p(beta),
                                       _p(y), _p(lo), _p(mean), _p(rstd), N, D, eps, _stream()))
    return x, y, lo, mean, rstd


def layernorm_bwd(dout, x, gamma, mean, rstd, dresid=None):
    """LayerNormBackward (src/tensor.cpp:324-359), plus dresid if given."""
    lib = _lib.load()
    _req(x, "x")
    _req(dout, "dout")
    D = x.shape[-1]
    N = x.numel() // D
    dx = torch.empty_like(x)
    dg = torch.empty(D, dtype=_f32, device=x.device)
    db = torch.empty(D, dtype=_f32, device=x.device)
    nb = lib.ns_layernorm_bwd_workspace_size(N, D)
    ws = _ws(nb, x.device)
    _lib.check(lib.ns_layernorm_bwd(_p(dout), _p(x), _p(gamma), _p(mean), _p(rstd), _p(dresid),
                                    _p(dx), _p(dg), _p(db), N, D, _p(ws), nb, _stream()))
    return dx, dg, db


def gelu_fwd(x):
    """GeluForward (src/tensor.cpp:428-443)."""
    _req(x, "x")
    y = torch.empty_like(x)
    _lib.check(_lib.load().ns_gelu_fwd(_p(x), _p(y), x.numel(), _stream()))
    return y


def gelu_fwd_lo(x):
    """(gelu(x), its tf32 lo part) in one pass (ns_gelu_fwd_lo)."""
    _req(x, "x")
    y = torch.empty_like(x)
    lo = torch.empty_like(x)
    _lib.check(_lib.load().ns_gelu_fwd_lo(_p(x), _p(y), _p(lo), x.numel(), _stream()))
    return y, lo


def gelu_bwd(dout, x):
    """GeluBackward (src/tensor.cpp:445-461)."""
    _req(x, "x")
    dx = torch.empty_like(x)
    _lib.check(_lib.load().ns_gelu_bwd(_p(dout), _p(x), _p(dx), x.numel(), _stream()))
    return dx


def add(a, b):
    """ElementwiseAdd (src/tensor.cpp:534-540)."""
    out = torch.empty_like(a)
    _lib.check(_lib.load().ns_add(_p(a), _p(b), _p(out), a.numel(), _stream()))
    return out


def cross_entropy(logits, targets, denom=None):
    """CrossEntropyLoss Forward+Backward (include/losses.h:34-86).

    Returns (loss tensor [1], dlogits, err flag tensor [1]).
    """
    lib = _lib.load()
    _req(logits, "logits")
    _req(targets, "targets", torch.int32)
    N, V = logits.shape
    loss = torch.empty(1, dtype=_f32, device=logits.device)
    d = torch.empty_like(logits)
    err = torch.zeros(1, dtype=torch.int32, device=logits.device)
    nb = lib.ns_cross_entropy_workspace_size(N, V)
    ws = _ws(nb, logits.device)
    _lib.check(lib.ns_cross_entropy(_p(logits), _p(targets), N, V, float(denom or N), _p(loss),
                                    _p(d), _p(err), _p(ws), nb, _stream()))
    return loss, d, err


def embedding_fwd(tokens, wte, wpe):
    """Embedding::Forward for wte and wpe plus the add (include/gpt.h:197-212)."""
    lib = _lib.load()
    _req(tokens, "tokens", torch.int32)
    B, T = tokens.shape
    V, C = wte.shape
    out = torch.empty((B, T, C), dtype=_f32, device=wte.device)
    err = torch.zeros(1, dtype=torch.int32, device=wte.device)
    _lib.check(lib.ns_embedding_fwd(_p(tokens), B, T, _p(wte), V, _p(wpe), wpe.shape[0], C,
                                    _p(out), _p(err), _stream()))
    return out, err


def embedding_bwd(tokens, dx, vocab, block, dwte=None, dwpe=None, accumulate_wte=False):
    """Embedding::Backward for wte and wpe (include/layers/embedding.h:61-80)."""
    lib = _lib.load()
    B, T = tokens.shape
    C = dx.shape[-1]
    if dwte is None:
        dwte = torch.zeros((vocab, C), dtype=_f32, device=dx.device)
    if dwpe is None:
        dwpe = torch.empty((block, C), dtype=_f32, device=dx.device)
    _lib.check(lib.ns_embedding_bwd(_p(tokens), B, T, _p(dx), vocab, block, C, _p(dwte),
                                    int(accumulate_wte), _p(dwpe), _stream()))
    return dwte, dwpe


def adamw_flat(params, grads, m, v, seg_offsets, seg_decay, lr, b1, b2, eps, bc1, bc2):
    """AdamW::Step (include/optimizers.h:206-234) over flat buffers."""
    import ctypes

    lib = _lib.load()
    n_seg = len(seg_decay)
    offs = (ctypes.c_int64 * (n_seg + 1))(*seg_offsets)
    dec = (ctypes.c_float * max(1, n_seg))(*seg_decay)
    _lib.check(lib.ns_adamw_flat(_p(params), _p(grads), _p(m), _p(v), params.numel(),
                                 ctypes.cast(offs, ctypes.c_void_p), ctypes.cast(dec, ctypes.c_void_p),
                                 n_seg, lr, b1, b2, eps, bc1, bc2, _stream()))


def sumsq(x):
    lib = _lib.load()
    out = torch.empty(1, dtype=_f32, device=x.device)
    nb = lib.ns_sumsq_workspace_size(x.numel())
    ws = _ws(nb, x.device)
    _lib.check(lib.ns_sumsq(_p(x), x.numel(), _p(out), _p(ws), nb, _stream()))
    return out


def clip_scale(x, sumsq_t, max_norm):
    _lib.check(_lib.load().ns_clip_scale(_p(x), x.numel(), _p(sumsq_t), max_norm, _stream()))


def conv2d_fwd(x, weight, bias, stride=1, pad=0):
    """Conv2D::Forward (include/layers/conv2d.h:211-266): x [B, IC, H, W],
    weight [OC, IC, k, k] -> y [B, OC, OH, OW]."""
    lib = _lib.load()
    _req(x, "x")
    _req(weight, "weight")
    B, IC, H, W = x.shape
    OC, _, k, _ = weight.shape
    OH, OW = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    y = torch.empty((B, OC, OH, OW), dtype=_f32, device=x.device)
    nb = lib.ns_conv2d_workspace_size(B, IC, H, W, OC, k, stride, pad)
    ws = _ws(nb, x.device)
    _lib.check(lib.ns_conv2d_fwd(_p(x), B, IC, H, W, _p(weight), _p(bias), OC, k, stride, pad,
                                 _p(y), _p(ws), nb, _stream()))
    return y


def conv2d_bwd(x, dy, weight, stride=1, pad=0, want_dx=True):
    """Conv2D::Backward (include/layers/conv2d.h:268-331): (dx, dweight, dbias)."""
    lib = _lib.load()
    for t, n in ((x, "x"), (dy, "dy"), (weight, "weight")):
        _req(t, n)
    B, IC, H, W = x.shape
    OC, _, k, _ = weight.shape
    dx = torch.empty_like(x) if want_dx else None
    dw = torch.empty_like(weight)
    db = torch.empty(OC, dtype=_f32, device=x.device)
    nb = lib.ns_conv2d_workspace_size(B, IC, H, W, OC, k, stride, pad)
    ws = _ws(nb, x.device)
    _lib.check(lib.ns_conv2d_bwd(_p(x), _p(dy), B, IC, H, W, _p(weight), OC, k, stride, pad,
                                 _p(dx), _p(dw), _p(db), _p(ws), nb, _stream()))
    return dx, dw, db


def _lstm_views(flat, IN, H):
    """Registration-order views (weight_ih [4H, IN], weight_hh [4H, H], bias_ih,
    bias_hh) of one cell's flat parameter (or gradient) tensor."""
    a, b = 4 * H * IN, 4 * H * IN + 4 * H * H
    return flat[:a].view(4 * H, IN), flat[a:b].view(4 * H, H), flat[b:b + 4 * H], flat[b + 4 * H:b + 8 * H]


def _lstm_struct(views):
    return _lib.ns_lstm_weights(*[v.data_ptr() for v in views])


def lstm_set_engine(engine: int) -> None:
    """0: the whole-sequence recurrence where it fits; 1: one launch per step."""
    _lib.check(_lib.load().ns_lstm_set_engine(engine))


def lstm_fwd_bwd(x, params, dout, H, bidir=False, want_dx=True):
    """LSTM / BiLSTM Forward then Backward (include/layers/lstm.h:320-664):
    x [T, B, IN], params flat in registration order -> (out, dx, grads flat)."""
    lib = _lib.load()
    _req(x, "x")
    T, B, IN = x.shape
    n1 = 4 * H * IN + 4 * H * H + 8 * H
    grads = torch.empty_like(params)
    dx = torch.empty_like(x) if want_dx else None
    if bidir:
        out = torch.empty((T, B, 2 * H), dtype=_f32, device=x.device)
        cache = torch.empty(lib.ns_bilstm_cache_floats(T, B, H), dtype=_f32, device=x.device)
        nb = lib.ns_bilstm_workspace_size(T, B, IN, H)
        ws = _ws(nb, x.device)
        wf, wr = (_lstm_struct(_lstm_views(params[o:o + n1], IN, H)) for o in (0, n1))
        gf, gr = (_lstm_struct(_lstm_views(grads[o:o + n1], IN, H)) for o in (0, n1))
        _lib.check(lib.ns_bilstm_fwd(_p(x), T, B, IN, H, wf, wr, _p(out), _p(cache), _p(ws), nb,
                                     _stream()))
        _lib.check(lib.ns_bilstm_bwd(_p(x), _p(dout), T, B, IN, H, wf, wr, _p(cache), _p(dx), gf,
                                     gr, _p(ws), nb, _stream()))
    else:
        out = torch.empty((T, B, H), dtype=_f32, device=x.device)
        cache = torch.empty(lib.ns_lstm_cache_floats(T, B, H), dtype=_f32, device=x.device)
        nb = lib.ns_lstm_workspace_size(T, B, IN, H)
        ws = _ws(nb, x.device)
        w = _lstm_struct(_lstm_views(params, IN, H))
        g = _lstm_struct(_lstm_views(grads, IN, H))
        _lib.check(lib.ns_lstm_fwd(_p(x), T, B, IN, H, w, _p(out), _p(cache), _p(ws), nb, _stream()))
        _lib.check(lib.ns_lstm_bwd(_p(x), _p(out), _p(dout), T, B, IN, H, w, _p(cache), _p(dx), g,
                                   _p(ws), nb, _stream()))
    return out, dx, grads
