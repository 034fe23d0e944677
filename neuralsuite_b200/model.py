"""Python face of the device GPT training step (the ns_gpt_* C ABI).

Mirrors the reference's GPTModel / CrossEntropyLoss / AdamW usage of
train_llm.cpp:176-228 and tools/parity/parity_gpt.cpp:55-97: construct with a
GPTConfig, load weights in GetParameters() order, run Forward -> loss ->
Backward -> AdamW.Step.  Parameters, gradients, optimizer state and
activations stay in HBM; torch tensors returned here are zero-copy views of
the library's buffers.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib


@dataclass
class GPTConfig:
    """include/gpt.h:33-39"""

    vocab_size: int = 54
    block_size: int = 64
    n_layer: int = 4
    n_head: int = 4
    n_embd: int = 128


class _DeviceView:
    """__cuda_array_interface__ over a device pointer owned by the library."""

    def __init__(self, ptr: int, n: int, dtype: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": dtype, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _device_tensor(ptr: int, n: int) -> torch.Tensor:
    return torch.as_tensor(_DeviceView(ptr, n), device="cuda")


def param_shapes(cfg: GPTConfig):
    """Shapes in registration order (include/gpt.h:143-149, 59-63)."""
    V, C = cfg.vocab_size, cfg.n_embd
    shapes = [(V, C), (cfg.block_size, C)]
    for _ in range(cfg.n_layer):
        shapes += [(C,), (C,), (C, 3 * C), (3 * C,), (C, C), (C,), (C,), (C,), (C, 4 * C), (4 * C,),
                   (4 * C, C), (C,)]
    return shapes + [(C,), (C,)]


def init_params(cfg: GPTConfig, rng: np.random.Generator, std: float = 0.02,
                ln_noise: float = 0.0) -> np.ndarray:
    """Flat float32 parameters with the reference's initialisation scheme:
    N(0, std) for wte, wpe and every Linear weight (include/layers/embedding.h:31,
    include/layers/linear.h:51-52, include/gpt.h:54-56), LayerNorm gamma = 1 and
    beta = 0 (include/layers/layernorm.h:31-32), Linear bias = 0
    (include/layers/linear.h:56).  ln_noise > 0 perturbs the 1-D parameters so
    tests exercise every gradient path."""
    shapes = param_shapes(cfg)
    parts = []
    L = cfg.n_layer
    for i, s in enumerate(shapes):
        n = int(np.prod(s))
        if len(s) == 2:
            parts.append((rng.standard_normal(n) * std).astype(np.float32))
            continue
        is_gamma = (2 <= i < 2 + 12 * L and (i - 2) % 12 in (0, 6)) or i == len(shapes) - 2
        base = np.ones(n, np.float32) if is_gamma else np.zeros(n, np.float32)
        if ln_noise:
            base = base + (rng.standard_normal(n) * ln_noise).astype(np.float32)
        parts.append(base.astype(np.float32))
    return np.concatenate(parts).astype(np.float32)


def nsf_save(cfg: GPTConfig, flat, path: str) -> None:
    """Flat host parameters (registration order) to an NSF file (no GPU)."""
    lib = _lib.load()
    a = np.ascontiguousarray(np.asarray(flat, dtype=np.float32))
    c = _lib.ns_gpt_config(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd, 1)
    _lib.check(lib.ns_nsf_save_gpt(ctypes.byref(c), a.ctypes.data, str(path).encode()))


def nsf_load(cfg: GPTConfig, path: str) -> np.ndarray:
    """NSF file to flat host parameters, checked against cfg (no GPU)."""
    lib = _lib.load()
    n = sum(int(np.prod(s)) for s in param_shapes(cfg))
    out = np.zeros(n, np.float32)
    c = _lib.ns_gpt_config(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd, 1)
    _lib.check(lib.ns_nsf_load_gpt(ctypes.byref(c), str(path).encode(), out.ctypes.data))
    return out


def plan_buckets(cfg: GPTConfig, bucket_floats: int = 0):
    """Gradient all-reduce buckets [(begin, end), ...] in launch order (host only)."""
    lib = _lib.load()
    c = _lib.ns_gpt_config(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd, 1)
    n = lib.ns_gpt_plan_buckets(ctypes.byref(c), bucket_floats, None, None, 0)
    b = (ctypes.c_int64 * max(n, 1))()
    e = (ctypes.c_int64 * max(n, 1))()
    lib.ns_gpt_plan_buckets(ctypes.byref(c), bucket_floats, b, e, n)
    return [(int(b[i]), int(e[i])) for i in range(n)]


class GPTModel:
    """Device GPTModel + CrossEntropyLoss + AdamW (include/gpt.h:136-327,
    include/losses.h:32-91, include/optimizers.h:143-253)."""

    def __init__(self, cfg: GPTConfig, max_batch: int):
        if cfg.n_head <= 0 or cfg.n_embd % cfg.n_head != 0:
            raise ValueError(f"n_embd ({cfg.n_embd}) must be divisible by n_head ({cfg.n_head})")
        self.lib = _lib.load()
        self.cfg = cfg
        self.max_batch = max_batch
        c = _lib.ns_gpt_config(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd,
                               max_batch)
        h = ctypes.c_void_p()
        _lib.check(self.lib.ns_gpt_create(ctypes.byref(c), ctypes.byref(h)))
        self.h = h
        self.n_params = int(self.lib.ns_gpt_num_params(self.h))
        self.n_tensors = int(self.lib.ns_gpt_num_tensors(self.h))
        self._comm = None
        self._tok = None
        self._tgt = None
        self.world = 1

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            self.lib.ns_gpt_destroy(h)
            self.h = None

    # ------------------------------------------------------------ parameters
    def tensor_numel(self, i):
        return int(self.lib.ns_gpt_tensor_numel(self.h, i))

    def tensor_rank(self, i):
        return int(self.lib.ns_gpt_tensor_rank(self.h, i))

    def tensor_offset(self, i):
        return int(self.lib.ns_gpt_tensor_offset(self.h, i))

    def params(self) -> torch.Tensor:
        """Flat device view of every parameter (GetParameters() order)."""
        return _device_tensor(self.lib.ns_gpt_params(self.h), self.n_params)

    def grads(self) -> torch.Tensor:
        """Flat device view of every gradient (GetGradients() order)."""
        return _device_tensor(self.lib.ns_gpt_grads(self.h), self.n_params)

    def set_params(self, flat) -> None:
        src = torch.as_tensor(np.asarray(flat, dtype=np.float32) if not torch.is_tensor(flat) else flat)
        if src.numel() != self.n_params:
            raise ValueError(f"expected {self.n_params} parameters, got {src.numel()}")
        self.params().copy_(src.reshape(-1).to(torch.float32))
        torch.cuda.synchronize()

    def get_params(self) -> np.ndarray:
        torch.cuda.synchronize()
        return self.params().cpu().numpy().copy()

    def get_grads(self) -> np.ndarray:
        torch.cuda.synchronize()
        return self.grads().cpu().numpy().copy()

    def logits(self, B: int, T: int) -> torch.Tensor:
        return _device_tensor(self.lib.ns_gpt_logits(self.h), B * T * self.cfg.vocab_size).view(
            B, T, self.cfg.vocab_size)

    def loss_tensor(self) -> torch.Tensor:
        return _device_tensor(self.lib.ns_gpt_loss(self.h), 1)

    # ------------------------------------------------------------ inputs
    def _ids(self, x, what, limit) -> torch.Tensor:
        """Token ids as a contiguous int32 device tensor.  Host input is
        validated first, which is where the reference's std::out_of_range
        (include/layers/embedding.h:45-49) comes from."""
        if torch.is_tensor(x) and x.is_cuda:
            return x.to(torch.int32).contiguous()
        a = np.asarray(x)
        ai = a.astype(np.int64)  # the reference truncates float ids (embedding.h:43)
        if ai.size and (ai.min() < 0 or ai.max() >= limit):
            raise IndexError(f"{what} id outside [0, {limit})")
        return torch.as_tensor(ai.astype(np.int32), device="cuda")

    # ------------------------------------------------------------ the step
    def forward(self, idx) -> torch.Tensor:
        """GPTModel::Forward (include/gpt.h:192-232); returns logits [B, T, V]."""
        t = self._ids(idx, "token", self.cfg.vocab_size)
        B, T = t.shape
        if T > self.cfg.block_size:
            raise IndexError("sequence longer than block_size")
        self._tok = t
        _lib.check(self.lib.ns_gpt_forward(self.h, t.data_ptr(), B, T, self._stream()))
        self._BT = (B, T)
        return self.logits(B, T)

    def loss_backward(self, targets) -> torch.Tensor:
        """CrossEntropyLoss::Forward + ::Backward (include/losses.h:34-86)."""
        tg = self._ids(targets, "target", self.cfg.vocab_size).reshape(-1)
        self._tgt = tg
        _lib.check(self.lib.ns_gpt_loss_backward(self.h, tg.data_ptr(), self._stream()))
        return self.loss_tensor()

    def backward(self) -> None:
        """GPTModel::Backward (include/gpt.h:234-272); gradients overwritten."""
        _lib.check(self.lib.ns_gpt_backward(self.h, self._stream()))

    def fwd_bwd(self, idx, targets):
        """Forward -> CrossEntropy -> Backward (tools/parity/parity_gpt.cpp:86-97).
        Returns (loss, logits numpy)."""
        logits = self.forward(idx)
        loss = self.loss_backward(targets)
        self.backward()
        torch.cuda.synchronize()
        return float(loss.item()), logits.cpu().numpy()

    def adamw_init(self, lr=1e-3, b1=0.9, b2=0.95, eps=1e-8, wd=0.01):
        """AdamW(params, lr, b1, b2, eps, wd) (include/optimizers.h:148-162)."""
        _lib.check(self.lib.ns_gpt_adamw_init(self.h, lr, b1, b2, eps, wd))

    def adamw_set_lr(self, lr):
        _lib.check(self.lib.ns_gpt_adamw_set_lr(self.h, lr))

    def adamw_step(self):
        _lib.check(self.lib.ns_gpt_adamw_step(self.h, self._stream()))

    def clip_gradients(self, max_norm=1.0):
        _lib.check(self.lib.ns_gpt_clip_gradients(self.h, max_norm, self._stream()))

    def train_step(self, tokens: torch.Tensor, targets: torch.Tensor, max_norm: float = 0.0,
                   read_loss: bool = True):
        """Forward, loss, backward (+ all-reduce), optional clip, AdamW step, on
        device int32 token / target tensors.  Returns the (global mean) loss
        when read_loss, else None without synchronising."""
        B, T = tokens.shape
        out = ctypes.c_float(0.0)
        _lib.check(self.lib.ns_gpt_train_step(self.h, tokens.data_ptr(), targets.data_ptr(), B, T,
                                              max_norm, ctypes.byref(out) if read_loss else None,
                                              self._stream()))
        return float(out.value) if read_loss else None

    # ------------------------------------------------------------ checkpoints
    def save_weights(self, path: str) -> None:
        """GPTModel::SaveWeights (include/gpt.h:293-300): an NSF file the
        reference reads."""
        _lib.check(self.lib.ns_gpt_save_weights(self.h, str(path).encode(), self._stream()))

    def load_weights(self, path: str) -> None:
        """GPTModel::LoadWeights (include/gpt.h:302-306); raises ValueError with
        the reason (wrong architecture, truncated, corrupt) and leaves the
        parameters unchanged."""
        _lib.check(self.lib.ns_gpt_load_weights(self.h, str(path).encode(), self._stream()))

    def save_optimizer(self, path: str) -> None:
        """AdamW moments, step count and hyper-parameters (NSF)."""
        _lib.check(self.lib.ns_gpt_save_optimizer(self.h, str(path).encode(), self._stream()))

    def load_optimizer(self, path: str) -> None:
        _lib.check(self.lib.ns_gpt_load_optimizer(self.h, str(path).encode(), self._stream()))

    # ------------------------------------------------------------ data parallel
    def set_comm(self, comm, world: int, bucket_floats: int = 0):
        _lib.check(self.lib.ns_gpt_set_comm(self.h, comm.handle if comm else None, world,
                                            bucket_floats))
        self._comm = comm
        self.world = world if comm else 1

    def set_comm_timing(self, enable: bool = True) -> None:
        """Record, in every backward, when the gradient all-reduces start and
        end and when the backward's own work ends (needs world > 1)."""
        _lib.check(self.lib.ns_gpt_set_comm_timing(self.h, 1 if enable else 0))

    def comm_times(self):
        """(exposed_ms, span_ms) of the last backward: the time the compute
        stream waited for the all-reduces after its backward, and the time
        from the first bucket's start to the last one's end."""
        exposed, span = ctypes.c_float(), ctypes.c_float()
        _lib.check(self.lib.ns_gpt_comm_times(self.h, ctypes.byref(exposed), ctypes.byref(span)))
        return float(exposed.value), float(span.value)

    @staticmethod
    def _stream():
        return torch.cuda.current_stream().cuda_stream


class Decoder:
    """KV-cache decoding of B sequences in lockstep on a GPTModel
    (GPTModel::ForwardWithKVCache / ClearKVCache, include/gpt.h:153-190)."""

    def __init__(self, model: GPTModel, max_batch: int = 1):
        self.model = model
        self.lib = model.lib
        h = ctypes.c_void_p()
        _lib.check(self.lib.ns_gpt_decoder_create(model.h, max_batch, ctypes.byref(h)))
        self.h = h
        self.err = torch.zeros(1, dtype=torch.int32, device="cuda")

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            self.lib.ns_gpt_decoder_destroy(h)
            self.h = None

    def clear(self):
        _lib.check(self.lib.ns_gpt_decoder_clear(self.h))

    def __len__(self):
        return int(self.lib.ns_gpt_decoder_length(self.h))

    def step(self, tokens, pos: int, out: torch.Tensor = None) -> torch.Tensor:
        """One token per sequence at position pos -> logits [B, V] (device)."""
        t = self.model._ids(tokens, "token", self.model.cfg.vocab_size).reshape(-1)
        B = t.numel()
        if out is None:
            out = torch.empty(B, self.model.cfg.vocab_size, device="cuda")
        _lib.check(self.lib.ns_gpt_decode_step(self.h, t.data_ptr(), B, pos, out.data_ptr(),
                                               self.err.data_ptr(), GPTModel._stream()))
        return out

    def prefill(self, tokens) -> torch.Tensor:
        """Prompt tokens [B, T] through the batched forward; fills the cache
        and returns the last position's logits [B, V]."""
        t = self.model._ids(tokens, "token", self.model.cfg.vocab_size)
        B, T = t.shape
        out = torch.empty(B, self.model.cfg.vocab_size, device="cuda")
        _lib.check(self.lib.ns_gpt_decoder_prefill(self.h, t.data_ptr(), B, T, out.data_ptr(),
                                                   GPTModel._stream()))
        return out

    def check(self):
        """Raises IndexError if a token of an earlier step was out of range."""
        if int(self.err.item()):
            self.err.zero_()
            raise IndexError("a decoded token id is outside [0, vocab_size)")


class UNet:
    """The diffusion U-Net training step on the device (ns_unet_*): Conv2D,
    ResidualBlock, LayerNormLayer and MSELoss of the reference wired as a
    two-level U-Net with nearest-neighbour upsampling."""

    def __init__(self, in_channels=3, base_channels=64, image_size=64, max_batch=32):
        self.lib = _lib.load()
        c = _lib.ns_unet_config(in_channels, base_channels, image_size, max_batch)
        h = ctypes.c_void_p()
        _lib.check(self.lib.ns_unet_create(ctypes.byref(c), ctypes.byref(h)))
        self.h = h
        self.in_channels, self.image_size, self.max_batch = in_channels, image_size, max_batch
        self.n_params = int(self.lib.ns_unet_num_params(h))
        self.n_tensors = int(self.lib.ns_unet_num_tensors(h))
        self.world = 1

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            self.lib.ns_unet_destroy(h)
            self.h = None

    def params(self) -> torch.Tensor:
        return _device_tensor(self.lib.ns_unet_params(self.h), self.n_params)

    def grads(self) -> torch.Tensor:
        return _device_tensor(self.lib.ns_unet_grads(self.h), self.n_params)

    def set_params(self, flat) -> None:
        src = torch.as_tensor(np.asarray(flat, dtype=np.float32))
        if src.numel() != self.n_params:
            raise ValueError(f"expected {self.n_params} parameters, got {src.numel()}")
        self.params().copy_(src.reshape(-1))
        torch.cuda.synchronize()

    def get_params(self) -> np.ndarray:
        torch.cuda.synchronize()
        return self.params().cpu().numpy().copy()

    def get_grads(self) -> np.ndarray:
        torch.cuda.synchronize()
        return self.grads().cpu().numpy().copy()

    def fwd_bwd(self, x, target):
        """Forward -> MSELoss -> Backward; returns (loss, prediction numpy)."""
        xd = torch.as_tensor(np.asarray(x, np.float32), device="cuda").contiguous()
        td = torch.as_tensor(np.asarray(target, np.float32), device="cuda").contiguous()
        B = xd.shape[0]
        s = GPTModel._stream()
        _lib.check(self.lib.ns_unet_forward(self.h, xd.data_ptr(), B, s))
        _lib.check(self.lib.ns_unet_loss_backward(self.h, td.data_ptr(), s))
        _lib.check(self.lib.ns_unet_backward(self.h, s))
        torch.cuda.synchronize()
        n = B * self.in_channels * self.image_size ** 2
        out = _device_tensor(self.lib.ns_unet_output(self.h), n).cpu().numpy()
        loss = float(_device_tensor(self.lib.ns_unet_loss(self.h), 1).item()) / self.world
        return loss, out.reshape(B, self.in_channels, self.image_size, self.image_size)

    def adamw_init(self, lr=1e-3, b1=0.9, b2=0.95, eps=1e-8, wd=0.01):
        _lib.check(self.lib.ns_unet_adamw_init(self.h, lr, b1, b2, eps, wd))

    def adamw_step(self):
        _lib.check(self.lib.ns_unet_adamw_step(self.h, GPTModel._stream()))

    def train_step(self, x: torch.Tensor, target: torch.Tensor, read_loss: bool = True):
        out = ctypes.c_float(0.0)
        _lib.check(self.lib.ns_unet_train_step(self.h, x.data_ptr(), target.data_ptr(), x.shape[0],
                                               ctypes.byref(out) if read_loss else None,
                                               GPTModel._stream()))
        return float(out.value) if read_loss else None

    def set_comm(self, comm, world: int):
        _lib.check(self.lib.ns_unet_set_comm(self.h, comm.handle if comm else None, world))
        self.world = world if comm else 1


class Comm:
    """NCCL communicator of the C ABI; the unique id travels over an existing
    torch.distributed process group (plumbing only)."""

    def __init__(self, rank: int, world: int, group=None):
        import torch.distributed as dist

        lib = _lib.load()
        buf = (ctypes.c_uint8 * 128)()
        if rank == 0:
            _lib.check(lib.ns_comm_unique_id(buf))
        obj = [bytes(buf) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(obj[0])
        h = ctypes.c_void_p()
        _lib.check(lib.ns_comm_init(uid, world, rank, ctypes.byref(h)))
        self.handle = h
        self.rank, self.world = rank, world
        self.lib = lib

    def allreduce_(self, t: torch.Tensor):
        _lib.check(self.lib.ns_comm_allreduce_sum(self.handle, t.data_ptr(), t.numel(),
                                                  torch.cuda.current_stream().cuda_stream))

    def check(self):
        _lib.check(self.lib.ns_comm_check(self.handle))

    def destroy(self):
        if self.handle:
            self.lib.ns_comm_destroy(self.handle)
            self.handle = None
