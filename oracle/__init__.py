"""Test infrastructure: the CPU oracle for the GPT training step. NOT product code.

Two interchangeable checkers behind one Python interface:

* ``port()`` -- ``libns_oracle.so``, the plain-C restatement in ``ns_oracle.c``.
* ``ref()``  -- ``_ref/libnsref.so``, the NeuralSuite reference itself (its
  ``src/tensor.cpp`` and headers compiled by ``oracle/Makefile``), driven
  through ``ref_harness.cpp``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` import this package, and only as the checker / CPU baseline: the
CUDA product path never routes through it.

All arrays are float32 numpy arrays in the reference's layouts (row-major,
token ids as floats).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "libns_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libnsref.so")

_f = ctypes.c_float
_i = ctypes.c_int
_p = ctypes.c_void_p
_ll = ctypes.c_longlong


def build(ref: bool = True) -> None:
    """Compile the C port (always) and the reference harness (if its sources exist)."""
    targets = ["port"]
    if ref and os.path.isdir(os.environ.get("NS_REFERENCE", "/root/reference")):
        targets.append("ref")
    env = dict(os.environ)
    if "NS_REFERENCE" in os.environ:
        env["REF"] = os.environ["NS_REFERENCE"]
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True, env=env)


def _ptr(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(_p)


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


class OracleError(RuntimeError):
    pass


class _Base:
    """Common numpy-facing API; subclasses bind the symbol prefix."""

    prefix = ""
    so_path = ""

    def __init__(self):
        if not os.path.exists(self.so_path):
            raise OracleError(f"oracle library missing: {self.so_path} (run oracle.build())")
        self.lib = ctypes.CDLL(self.so_path)

    def _fn(self, name, argtypes, restype=_i):
        fn = getattr(self.lib, self.prefix + name)
        fn.argtypes = argtypes
        fn.restype = restype
        return fn

    # -- primitives ------------------------------------------------------
    def matmul(self, A, B):
        A, B = f32(A), f32(B)
        M, K = A.shape
        K2, N = B.shape
        assert K == K2
        C = np.zeros((M, N), np.float32)
        self._call("matmul", [_p, _p, _p, _i, _i, _i], _ptr(A), _ptr(B), _ptr(C), M, K, N)
        return C

    def layernorm_fwd(self, x, gamma, beta, eps=1e-5):
        x, gamma, beta = f32(x), f32(gamma), f32(beta)
        D = x.shape[-1]
        N = x.size // D
        out = np.zeros_like(x)
        mean = np.zeros(N, np.float32)
        rstd = np.zeros(N, np.float32)
        self._call("layernorm_fwd", [_p] * 6 + [_i, _i, _f], _ptr(x), _ptr(gamma), _ptr(beta),
                   _ptr(out), _ptr(mean), _ptr(rstd), N, D, eps)
        return out, mean, rstd

    def layernorm_bwd(self, dout, x, gamma, mean, rstd):
        dout, x, gamma, mean, rstd = map(f32, (dout, x, gamma, mean, rstd))
        D = x.shape[-1]
        N = x.size // D
        dx = np.zeros_like(x)
        dg = np.zeros(D, np.float32)
        db = np.zeros(D, np.float32)
        self._call("layernorm_bwd", [_p] * 8 + [_i, _i], _ptr(dout), _ptr(x), _ptr(gamma),
                   _ptr(mean), _ptr(rstd), _ptr(dx), _ptr(dg), _ptr(db), N, D)
        return dx, dg, db

    def cross_entropy(self, logits, targets):
        logits, targets = f32(logits), f32(targets)
        N, V = logits.shape
        d = np.zeros_like(logits)
        return self._ce(logits, targets, N, V, d), d

    def gpt(self, vocab, block, n_layer, n_head, n_embd):
        return self._gpt_cls(self, vocab, block, n_layer, n_head, n_embd)


class _PortGpt:
    def __init__(self, o, V, block, L, H, C):
        self.o = o
        lib = o.lib
        lib.nso_gpt_create.restype = _p
        lib.nso_gpt_create.argtypes = [_i] * 5
        self.h = lib.nso_gpt_create(V, block, L, H, C)
        if not self.h:
            raise ValueError("n_embd must be divisible by n_head")
        self.V, self.block, self.L, self.H, self.C = V, block, L, H, C
        for name, res, args in [("nso_gpt_num_tensors", _i, [_p]),
                                ("nso_gpt_tensor_numel", ctypes.c_int64, [_p, _i]),
                                ("nso_gpt_tensor_rank", _i, [_p, _i]),
                                ("nso_gpt_num_params", ctypes.c_int64, [_p]),
                                ("nso_gpt_params", ctypes.POINTER(_f), [_p]),
                                ("nso_gpt_grads", ctypes.POINTER(_f), [_p]),
                                ("nso_gpt_fwd_bwd", _i, [_p, _p, _p, _i, _i, _p, _p]),
                                ("nso_gpt_clip_gradients", _f, [_p, _f]),
                                ("nso_gpt_adamw_init", None, [_p, _f, _f, _f, _f, _f]),
                                ("nso_gpt_adamw_set_lr", None, [_p, _f]),
                                ("nso_gpt_adamw_step", None, [_p]),
                                ("nso_gpt_destroy", None, [_p])]:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        self.n = lib.nso_gpt_num_params(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            self.o.lib.nso_gpt_destroy(self.h)
            self.h = None

    def num_tensors(self):
        return self.o.lib.nso_gpt_num_tensors(self.h)

    def tensor_numel(self, i):
        return int(self.o.lib.nso_gpt_tensor_numel(self.h, i))

    def tensor_rank(self, i):
        return int(self.o.lib.nso_gpt_tensor_rank(self.h, i))

    def num_params(self):
        return int(self.n)

    def set_params(self, flat):
        flat = f32(flat)
        assert flat.size == self.n
        ctypes.memmove(self.o.lib.nso_gpt_params(self.h), flat.ctypes.data, flat.nbytes)

    def get_params(self):
        return np.ctypeslib.as_array(self.o.lib.nso_gpt_params(self.h), (self.n,)).copy()

    def get_grads(self):
        return np.ctypeslib.as_array(self.o.lib.nso_gpt_grads(self.h), (self.n,)).copy()

    def fwd_bwd(self, idx, targets):
        idx, targets = f32(idx), f32(targets)
        B, T = idx.shape
        loss = _f(0.0)
        logits = np.zeros((B, T, self.V), np.float32)
        rc = self.o.lib.nso_gpt_fwd_bwd(self.h, _ptr(idx), _ptr(targets), B, T,
                                        ctypes.cast(ctypes.byref(loss), _p), _ptr(logits))
        if rc != 0:
            raise IndexError("token or position out of range")
        return float(loss.value), logits

    def clip_gradients(self, max_norm=1.0):
        return float(self.o.lib.nso_gpt_clip_gradients(self.h, max_norm))

    def adamw_init(self, lr=1e-3, b1=0.9, b2=0.95, eps=1e-8, wd=0.01):
        self.o.lib.nso_gpt_adamw_init(self.h, lr, b1, b2, eps, wd)

    def adamw_set_lr(self, lr):
        self.o.lib.nso_gpt_adamw_set_lr(self.h, lr)

    def adamw_step(self):
        self.o.lib.nso_gpt_adamw_step(self.h)


class _RefGpt(_PortGpt):
    def __init__(self, o, V, block, L, H, C):  # noqa: D401 - same interface as the port
        self.o = o
        lib = o.lib
        lib.nsref_gpt_create.restype = _p
        lib.nsref_gpt_create.argtypes = [_i] * 5
        self.h = lib.nsref_gpt_create(V, block, L, H, C)
        if not self.h:
            raise ValueError(lib.nsref_last_error().decode() if False else "bad GPT config")
        self.V, self.block, self.L, self.H, self.C = V, block, L, H, C
        for name, res, args in [("nsref_gpt_num_tensors", _i, [_p]),
                                ("nsref_gpt_tensor_numel", _ll, [_p, _i]),
                                ("nsref_gpt_tensor_rank", _i, [_p, _i]),
                                ("nsref_gpt_set_params", None, [_p, _p]),
                                ("nsref_gpt_get_params", None, [_p, _p]),
                                ("nsref_gpt_get_grads", None, [_p, _p]),
                                ("nsref_gpt_fwd_bwd", _i, [_p, _p, _p, _i, _i, _p, _p]),
                                ("nsref_gpt_clip_gradients", _f, [_p, _f]),
                                ("nsref_gpt_adamw_init", _i, [_p, _f, _f, _f, _f, _f]),
                                ("nsref_gpt_adamw_set_lr", None, [_p, _f]),
                                ("nsref_gpt_adamw_step", _i, [_p]),
                                ("nsref_gpt_destroy", None, [_p]),
                                ("nsref_gpt_decode", _i, [_p, _i, _i, _p]),
                                ("nsref_gpt_clear_kv", None, [_p]),
                                ("nsref_last_error", ctypes.c_char_p, [])]:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        self.n = sum(self.tensor_numel(i) for i in range(self.num_tensors()))

    def __del__(self):
        if getattr(self, "h", None):
            self.o.lib.nsref_gpt_destroy(self.h)
            self.h = None

    def num_tensors(self):
        return self.o.lib.nsref_gpt_num_tensors(self.h)

    def tensor_numel(self, i):
        return int(self.o.lib.nsref_gpt_tensor_numel(self.h, i))

    def tensor_rank(self, i):
        return int(self.o.lib.nsref_gpt_tensor_rank(self.h, i))

    def set_params(self, flat):
        flat = f32(flat)
        assert flat.size == self.n
        self.o.lib.nsref_gpt_set_params(self.h, _ptr(flat))

    def get_params(self):
        out = np.zeros(self.n, np.float32)
        self.o.lib.nsref_gpt_get_params(self.h, _ptr(out))
        return out

    def get_grads(self):
        out = np.zeros(self.n, np.float32)
        self.o.lib.nsref_gpt_get_grads(self.h, _ptr(out))
        return out

    def fwd_bwd(self, idx, targets):
        idx, targets = f32(idx), f32(targets)
        B, T = idx.shape
        loss = _f(0.0)
        logits = np.zeros((B, T, self.V), np.float32)
        rc = self.o.lib.nsref_gpt_fwd_bwd(self.h, _ptr(idx), _ptr(targets), B, T,
                                          ctypes.cast(ctypes.byref(loss), _p), _ptr(logits))
        if rc == 3:
            raise IndexError(self.o.lib.nsref_last_error().decode())
        if rc != 0:
            raise OracleError(self.o.lib.nsref_last_error().decode())
        return float(loss.value), logits

    def clip_gradients(self, max_norm=1.0):
        return float(self.o.lib.nsref_gpt_clip_gradients(self.h, max_norm))

    def adamw_init(self, lr=1e-3, b1=0.9, b2=0.95, eps=1e-8, wd=0.01):
        self.o.lib.nsref_gpt_adamw_init(self.h, lr, b1, b2, eps, wd)

    def adamw_set_lr(self, lr):
        self.o.lib.nsref_gpt_adamw_set_lr(self.h, lr)

    def adamw_step(self):
        self.o.lib.nsref_gpt_adamw_step(self.h)

    def decode(self, token, pos):
        """ForwardWithKVCache(token, pos) -> logits [V] (include/gpt.h:159-190)."""
        out = np.zeros(self.V, np.float32)
        rc = self.o.lib.nsref_gpt_decode(self.h, int(token), int(pos), _ptr(out))
        if rc == 3:
            raise IndexError(self.o.lib.nsref_last_error().decode())
        if rc != 0:
            raise OracleError(self.o.lib.nsref_last_error().decode())
        return out

    def clear_kv(self):
        self.o.lib.nsref_gpt_clear_kv(self.h)


class Port(_Base):
    """The plain-C restatement (ns_oracle.c)."""

    prefix = "nso_"
    so_path = PORT_SO
    _gpt_cls = _PortGpt

    def _call(self, name, argtypes, *args):
        fn = self._fn(name, argtypes, None)
        fn(*args)

    def _ce(self, logits, targets, N, V, d):
        fn = self._fn("cross_entropy", [_p, _p, _i, _i, _p], _f)
        return float(fn(_ptr(logits), _ptr(targets), N, V, _ptr(d)))

    def gelu_fwd(self, x):
        x = f32(x)
        y = np.zeros_like(x)
        self._fn("gelu_fwd", [_p, _p, ctypes.c_int64], None)(_ptr(x), _ptr(y), x.size)
        return y

    def gelu_bwd(self, dout, x):
        dout, x = f32(dout), f32(x)
        dx = np.zeros_like(x)
        self._fn("gelu_bwd", [_p, _p, _p, ctypes.c_int64], None)(_ptr(dout), _ptr(x), _ptr(dx),
                                                                 x.size)
        return dx

    def causal_softmax(self, s):
        s = f32(s)
        b, T, _ = s.shape
        out = np.zeros_like(s)
        self._fn("causal_softmax", [_p, _p, _i, _i], None)(_ptr(s), _ptr(out), b, T)
        return out

    def embedding(self, weight, idx, dout=None):
        weight, idx = f32(weight), f32(idx)
        num, dim = weight.shape
        B, T = idx.shape
        out = np.zeros((B, T, dim), np.float32)
        rc = self._fn("embedding_fwd", [_p, _i, _i, _p, _i, _p], _i)(
            _ptr(weight), num, dim, _ptr(idx), B * T, _ptr(out))
        if rc != 0:
            raise IndexError("token out of range")
        dw = None
        if dout is not None:
            dout = f32(dout)
            dw = np.zeros_like(weight)
            self._fn("embedding_bwd", [_p, _i, _i, _p, _i, _i, _p], None)(
                _ptr(idx), B * T, B * T, _ptr(dout), dim, num, _ptr(dw))
        return out, dw

    def adamw_flat(self, params, grads, m, v, offsets, decay, lr, b1, b2, eps, step):
        """In place on float32 arrays params, m, v (optimizers.h:206-234)."""
        offs = np.ascontiguousarray(np.asarray(offsets, dtype=np.int64))
        dec = f32(decay)
        self._fn("adamw_flat", [_p] * 6 + [_i, _f, _f, _f, _f, _i], None)(
            _ptr(params), _ptr(f32(grads)), _ptr(m), _ptr(v), offs.ctypes.data_as(_p), _ptr(dec),
            len(dec), lr, b1, b2, eps, step)

    def mha(self, B, T, C, H, w_attn, b_attn, w_proj, b_proj, x, dout):
        args = list(map(f32, (w_attn, b_attn, w_proj, b_proj, x, dout)))
        y = np.zeros((B, T, C), np.float32)
        dx = np.zeros((B, T, C), np.float32)
        g = [np.zeros_like(a) for a in args[:4]]
        rc = self._fn("mha", [_i] * 4 + [_p] * 12, _i)(
            B, T, C, H, *[_ptr(a) for a in args], _ptr(y), _ptr(dx), *[_ptr(a) for a in g])
        if rc != 0:
            raise ValueError("n_embd must be divisible by n_head")
        return y, dx, g


class Ref(_Base):
    """The NeuralSuite reference compiled from its own sources (oracle/_ref)."""

    prefix = "nsref_"
    so_path = REF_SO
    _gpt_cls = _RefGpt

    def _call(self, name, argtypes, *args):
        fn = self._fn(name, argtypes, _i)
        rc = fn(*args)
        if rc != 0:
            err = self._fn("last_error", [], ctypes.c_char_p)().decode()
            if rc == 3:
                raise IndexError(err)
            if rc == 2:
                raise ValueError(err)
            raise OracleError(err)

    def set_threads(self, n):
        self._fn("set_threads", [_i], None)(n)

    def threads(self):
        return self._fn("threads", [], _i)()

    def _ce(self, logits, targets, N, V, d):
        loss = _f(0.0)
        self._call("cross_entropy", [_p, _p, _i, _i, _p, _p], _ptr(logits), _ptr(targets), N, V,
                   ctypes.cast(ctypes.byref(loss), _p), _ptr(d))
        return float(loss.value)

    def gelu_fwd(self, x):
        x = f32(x)
        y = np.zeros_like(x)
        self._call("gelu_fwd", [_p, _p, _i], _ptr(x), _ptr(y), x.size)
        return y

    def gelu_bwd(self, dout, x):
        dout, x = f32(dout), f32(x)
        dx = np.zeros_like(x)
        self._call("gelu_bwd", [_p, _p, _p, _i], _ptr(dout), _ptr(x), _ptr(dx), x.size)
        return dx

    def causal_softmax(self, s):
        s = f32(s)
        b, T, _ = s.shape
        out = np.zeros_like(s)
        self._call("causal_softmax", [_p, _p, _i, _i], _ptr(s), _ptr(out), b, T)
        return out

    def embedding(self, weight, idx, dout=None):
        weight, idx = f32(weight), f32(idx)
        num, dim = weight.shape
        B, T = idx.shape
        out = np.zeros((B, T, dim), np.float32)
        dw = np.zeros_like(weight) if dout is not None else None
        self._call("embedding", [_p, _i, _i, _p, _i, _i, _p, _p, _p], _ptr(weight), num, dim,
                   _ptr(idx), B, T, _ptr(f32(dout)) if dout is not None else None, _ptr(out),
                   _ptr(dw))
        return out, dw

    def mha(self, B, T, C, H, w_attn, b_attn, w_proj, b_proj, x, dout):
        args = list(map(f32, (w_attn, b_attn, w_proj, b_proj, x, dout)))
        y = np.zeros((B, T, C), np.float32)
        dx = np.zeros((B, T, C), np.float32)
        g = [np.zeros_like(a) for a in args[:4]]
        self._call("mha", [_i] * 4 + [_p] * 12, B, T, C, H, *[_ptr(a) for a in args], _ptr(y),
                   _ptr(dx), *[_ptr(a) for a in g])
        return y, dx, g

    def lstm(self, x, params, dout, hidden, bidir=False):
        """LSTM / BiLSTM Forward + Backward: (out, dx, grads), params and grads
        flat in registration order."""
        x, params, dout = f32(x), f32(params), f32(dout)
        T, B, IN = x.shape
        out = np.zeros((T, B, (2 if bidir else 1) * hidden), np.float32)
        dx = np.zeros_like(x)
        grads = np.zeros_like(params)
        self._call("lstm", [_i] * 5 + [_p] * 6, T, B, IN, hidden, int(bidir), _ptr(params),
                   _ptr(x), _ptr(dout), _ptr(out), _ptr(dx), _ptr(grads))
        return out, dx, grads

    def conv2d(self, x, weight, bias, stride, pad, dout=None):
        """Conv2D::Forward (+ ::Backward with dout): y, and (dx, dweight, dbias)."""
        x, weight, bias = f32(x), f32(weight), f32(bias)
        B, IC, H, W = x.shape
        OC, _, k, _ = weight.shape
        OH, OW = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
        y = np.zeros((B, OC, OH, OW), np.float32)
        dx, dw, db = np.zeros_like(x), np.zeros_like(weight), np.zeros_like(bias)
        self._call("conv2d", [_i] * 8 + [_p] * 8, B, IC, H, W, OC, k, stride, pad, _ptr(weight),
                   _ptr(bias), _ptr(x), _ptr(f32(dout)) if dout is not None else None, _ptr(y),
                   _ptr(dx), _ptr(dw), _ptr(db))
        return (y, dx, dw, db) if dout is not None else y


class RefUNet:
    """The diffusion U-Net built from the reference's Conv2D / ResidualBlock /
    LayerNormLayer / MSELoss / AdamW (ref_harness.cpp; only the nearest
    upsample is written there)."""

    def __init__(self, o, in_ch, base, hw):
        lib = o.lib
        for name, res, args in [("nsref_unet_create", _p, [_i, _i, _i]),
                                ("nsref_unet_destroy", None, [_p]),
                                ("nsref_unet_num_tensors", _i, [_p]),
                                ("nsref_unet_tensor_numel", _ll, [_p, _i]),
                                ("nsref_unet_set_params", None, [_p, _p]),
                                ("nsref_unet_get", None, [_p, _i, _p]),
                                ("nsref_unet_fwd_bwd", _i, [_p, _i, _p, _p, _p, _p]),
                                ("nsref_unet_adamw_init", _i, [_p, _f]),
                                ("nsref_unet_adamw_step", _i, [_p])]:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        self.o, self.lib = o, lib
        self.h = lib.nsref_unet_create(in_ch, base, hw)
        self.in_ch, self.hw = in_ch, hw
        self.n = sum(int(lib.nsref_unet_tensor_numel(self.h, i))
                     for i in range(lib.nsref_unet_num_tensors(self.h)))

    def __del__(self):
        if getattr(self, "h", None):
            self.lib.nsref_unet_destroy(self.h)
            self.h = None

    def tensor_sizes(self):
        return [int(self.lib.nsref_unet_tensor_numel(self.h, i))
                for i in range(self.lib.nsref_unet_num_tensors(self.h))]

    def set_params(self, flat):
        flat = f32(flat)
        assert flat.size == self.n
        self.lib.nsref_unet_set_params(self.h, _ptr(flat))

    def _get(self, grads):
        out = np.zeros(self.n, np.float32)
        self.lib.nsref_unet_get(self.h, grads, _ptr(out))
        return out

    def get_params(self):
        return self._get(0)

    def get_grads(self):
        return self._get(1)

    def fwd_bwd(self, x, target):
        x, target = f32(x), f32(target)
        loss = _f(0.0)
        out = np.zeros_like(x)
        rc = self.lib.nsref_unet_fwd_bwd(self.h, x.shape[0], _ptr(x), _ptr(target),
                                         ctypes.cast(ctypes.byref(loss), _p), _ptr(out))
        if rc != 0:
            raise OracleError(self.lib.nsref_last_error().decode())
        return float(loss.value), out

    def adamw_init(self, lr):
        self.lib.nsref_unet_adamw_init(self.h, lr)

    def adamw_step(self):
        self.lib.nsref_unet_adamw_step(self.h)


_port = None
_ref = None


def port() -> Port:
    global _port
    if _port is None:
        _port = Port()
    return _port


def ref() -> Ref:
    global _ref
    if _ref is None:
        _ref = Ref()
    return _ref


def ref_available() -> bool:
    return os.path.exists(REF_SO)
