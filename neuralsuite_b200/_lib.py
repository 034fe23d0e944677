"""ctypes binding of ``include/ns_b200.h`` (the C ABI of libns_b200.so).

The library is loaded lazily and must exist: there is no fallback path.  Torch
is imported first so that the library binds to the CUDA runtime torch already
loaded (one runtime instance: same current device, same streams).
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libns_b200.so")

c_int, c_float, c_void_p, c_size_t = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t
c_int64 = ctypes.c_int64
P = c_void_p

NS_OK = 0
NS_ERR_INVALID_ARGUMENT = 1
NS_ERR_OUT_OF_RANGE = 2
NS_ERR_CUDA = 3
NS_ERR_UNSUPPORTED = 4
NS_ERR_COMM = 5
NS_ERR_TIMEOUT = 6

EPI_STORE, EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESID, EPI_GELU_BWD = range(5)


class NsError(RuntimeError):
    """A non-OK ns_status (CUDA, comm, timeout, unsupported)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[ns_status {code}] {msg}")
        self.code = code


class ns_lstm_weights(ctypes.Structure):
    _fields_ = [("w_ih", c_void_p), ("w_hh", c_void_p), ("b_ih", c_void_p), ("b_hh", c_void_p)]


ns_lstm_grads = ns_lstm_weights  # same layout (four device pointers)


class ns_unet_config(ctypes.Structure):
    _fields_ = [("in_channels", c_int), ("base_channels", c_int), ("image_size", c_int),
                ("max_batch", c_int)]


class ns_gpt_config(ctypes.Structure):
    _fields_ = [("vocab_size", c_int), ("block_size", c_int), ("n_layer", c_int),
                ("n_head", c_int), ("n_embd", c_int), ("max_batch", c_int)]


# name -> (restype, argtypes); kept in the order of the header.
_SIGS = {
    "ns_last_error": (ctypes.c_char_p, []),
    "ns_version": (c_int, []),
    "ns_launch_count": (ctypes.c_longlong, []),
    "ns_device_supported": (c_int, []),
    "ns_gemm_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "ns_gemm": (c_int, [c_int, c_int, c_int, P, c_int, c_int, P, c_int, c_int, P, c_int, c_float,
                        c_int, P, P, P, P, c_size_t, P]),
    "ns_gemm_lo": (c_int, [c_int, c_int, c_int, P, c_int, c_int, P, P, c_int, c_int, P, P, c_int,
                           c_float, c_int, P, P, P, P, c_size_t, P]),
    "ns_gemm_lo_out": (c_int, [c_int, c_int, c_int, P, c_int, c_int, P, P, c_int, c_int, P, P,
                               c_int, c_float, c_int, P, P, P, P, P, c_size_t, P]),
    "ns_split_lo": (c_int, [P, c_int, c_int, c_int, P, P]),
    "ns_gemm_set_engine": (c_int, [c_int]),
    "ns_kernel_health": (c_int, []),
    "ns_selftest_device_wait": (c_int, [c_int, P]),
    "ns_bias_grad_workspace_size": (c_size_t, [c_int, c_int]),
    "ns_bias_grad": (c_int, [P, c_int, c_int, P, P, c_size_t, P]),
    "ns_bias_grad_split": (c_int, [P, c_int, c_int, P, P, P, c_size_t, P]),
    "ns_bias_grad_split_gelu": (c_int, [P, P, c_int, c_int, P, P, P, c_size_t, P]),
    "ns_attn_fwd_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int]),
    "ns_attn_fwd": (c_int, [P, c_int, c_int, c_int, c_int, P, P, P, c_size_t, P]),
    "ns_attn_fwd_lo": (c_int, [P, P, c_int, c_int, c_int, c_int, P, P, P, P, c_size_t, P]),
    "ns_attn_set_engine": (c_int, [c_int]),
    "ns_attn_bwd_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int]),
    "ns_attn_bwd": (c_int, [P, P, P, P, c_int, c_int, c_int, c_int, P, P, c_size_t, P]),
    "ns_attn_bwd_lo": (c_int, [P, P, P, P, P, c_int, c_int, c_int, c_int, P, P, c_size_t, P]),
    "ns_layernorm_fwd": (c_int, [P, P, P, P, P, P, c_int, c_int, c_float, P]),
    "ns_layernorm_fwd_ex": (c_int, [P, P, P, P, P, P, P, P, P, P, c_int, c_int, c_float, P]),
    "ns_layernorm_bwd_workspace_size": (c_size_t, [c_int, c_int]),
    "ns_layernorm_bwd": (c_int, [P, P, P, P, P, P, P, P, P, c_int, c_int, P, c_size_t, P]),
    "ns_gelu_fwd": (c_int, [P, P, c_int64, P]),
    "ns_gelu_fwd_lo": (c_int, [P, P, P, c_int64, P]),
    "ns_gelu_bwd": (c_int, [P, P, P, c_int64, P]),
    "ns_add": (c_int, [P, P, P, c_int64, P]),
    "ns_cross_entropy_workspace_size": (c_size_t, [c_int, c_int]),
    "ns_cross_entropy": (c_int, [P, P, c_int, c_int, c_float, P, P, P, P, c_size_t, P]),
    "ns_cross_entropy_noalloc": (c_int, [P, P, c_int, c_int, c_float, P, P, P, P]),
    "ns_conv2d_workspace_size": (c_size_t, [c_int] * 8),
    "ns_conv2d_fwd": (c_int, [P, c_int, c_int, c_int, c_int, P, P, c_int, c_int, c_int, c_int, P,
                              P, c_size_t, P]),
    "ns_conv2d_bwd": (c_int, [P, P, c_int, c_int, c_int, c_int, P, c_int, c_int, c_int, c_int, P,
                              P, P, P, c_size_t, P]),
    "ns_lstm_cache_floats": (c_size_t, [c_int, c_int, c_int]),
    "ns_lstm_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int]),
    "ns_lstm_fwd": (c_int, [P, c_int, c_int, c_int, c_int, ns_lstm_weights, P, P, P, c_size_t, P]),
    "ns_lstm_bwd": (c_int, [P, P, P, c_int, c_int, c_int, c_int, ns_lstm_weights, P, P,
                            ns_lstm_weights, P, c_size_t, P]),
    "ns_bilstm_cache_floats": (c_size_t, [c_int, c_int, c_int]),
    "ns_bilstm_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int]),
    "ns_bilstm_fwd": (c_int, [P, c_int, c_int, c_int, c_int, ns_lstm_weights, ns_lstm_weights, P,
                              P, P, c_size_t, P]),
    "ns_bilstm_bwd": (c_int, [P, P, c_int, c_int, c_int, c_int, ns_lstm_weights, ns_lstm_weights,
                              P, P, ns_lstm_weights, ns_lstm_weights, P, c_size_t, P]),
    "ns_embedding_fwd": (c_int, [P, c_int, c_int, P, c_int, P, c_int, c_int, P, P, P]),
    "ns_embedding_bwd": (c_int, [P, c_int, c_int, P, c_int, c_int, c_int, P, c_int, P, P]),
    "ns_adamw_flat": (c_int, [P, P, P, P, c_int64, P, P, c_int, c_float, c_float, c_float,
                              c_float, c_float, c_float, P]),
    "ns_adamw_flat_device": (c_int, [P, P, P, P, c_int64, P, P, c_int, P, P]),
    "ns_sumsq_workspace_size": (c_size_t, [c_int64]),
    "ns_sumsq": (c_int, [P, c_int64, P, P, c_size_t, P]),
    "ns_clip_scale": (c_int, [P, c_int64, P, c_float, P]),
    "ns_comm_unique_id": (c_int, [P]),
    "ns_comm_init": (c_int, [P, c_int, c_int, P]),
    "ns_comm_allreduce_sum": (c_int, [P, P, c_int64, P]),
    "ns_comm_check": (c_int, [P]),
    "ns_comm_abort": (c_int, [P]),
    "ns_comm_destroy": (c_int, [P]),
    "ns_comm_selftest": (c_int, [c_int, ctypes.c_double, P]),
    "ns_gpt_save_weights": (c_int, [P, ctypes.c_char_p, P]),
    "ns_gpt_load_weights": (c_int, [P, ctypes.c_char_p, P]),
    "ns_nsf_save_gpt": (c_int, [P, P, ctypes.c_char_p]),
    "ns_nsf_load_gpt": (c_int, [P, ctypes.c_char_p, P]),
    "ns_gpt_save_optimizer": (c_int, [P, ctypes.c_char_p, P]),
    "ns_gpt_load_optimizer": (c_int, [P, ctypes.c_char_p, P]),
    "ns_gpt_decoder_create": (c_int, [P, c_int, P]),
    "ns_gpt_decoder_destroy": (c_int, [P]),
    "ns_gpt_decoder_clear": (c_int, [P]),
    "ns_gpt_decoder_length": (c_int, [P]),
    "ns_gpt_decoder_logits": (P, [P]),
    "ns_gpt_decode_step": (c_int, [P, P, c_int, c_int, P, P, P]),
    "ns_gpt_decoder_prefill": (c_int, [P, P, c_int, c_int, P, P]),
    "ns_unet_create": (c_int, [P, P]),
    "ns_unet_destroy": (c_int, [P]),
    "ns_unet_num_tensors": (c_int, [P]),
    "ns_unet_tensor_numel": (c_int64, [P, c_int]),
    "ns_unet_num_params": (c_int64, [P]),
    "ns_unet_params": (P, [P]),
    "ns_unet_grads": (P, [P]),
    "ns_unet_output": (P, [P]),
    "ns_unet_loss": (P, [P]),
    "ns_unet_forward": (c_int, [P, P, c_int, P]),
    "ns_unet_loss_backward": (c_int, [P, P, P]),
    "ns_unet_backward": (c_int, [P, P]),
    "ns_unet_adamw_init": (c_int, [P, c_float, c_float, c_float, c_float, c_float]),
    "ns_unet_adamw_step": (c_int, [P, P]),
    "ns_unet_train_step": (c_int, [P, P, P, c_int, P, P]),
    "ns_unet_set_comm": (c_int, [P, P, c_int]),
    "ns_gpt_create": (c_int, [P, P]),
    "ns_gpt_destroy": (c_int, [P]),
    "ns_gpt_num_tensors": (c_int, [P]),
    "ns_gpt_tensor_numel": (c_int64, [P, c_int]),
    "ns_gpt_tensor_rank": (c_int, [P, c_int]),
    "ns_gpt_tensor_offset": (c_int64, [P, c_int]),
    "ns_gpt_num_params": (c_int64, [P]),
    "ns_gpt_params": (P, [P]),
    "ns_gpt_grads": (P, [P]),
    "ns_gpt_logits": (P, [P]),
    "ns_gpt_loss": (P, [P]),
    "ns_gpt_forward": (c_int, [P, P, c_int, c_int, P]),
    "ns_gpt_loss_backward": (c_int, [P, P, P]),
    "ns_gpt_backward": (c_int, [P, P]),
    "ns_gpt_adamw_init": (c_int, [P, c_float, c_float, c_float, c_float, c_float]),
    "ns_gpt_adamw_set_lr": (c_int, [P, c_float]),
    "ns_gpt_adamw_step": (c_int, [P, P]),
    "ns_gpt_clip_gradients": (c_int, [P, c_float, P]),
    "ns_gpt_train_step": (c_int, [P, P, P, c_int, c_int, c_float, P, P]),
    "ns_gpt_set_comm": (c_int, [P, P, c_int, c_int64]),
    "ns_gpt_plan_buckets": (c_int, [P, c_int64, P, P, c_int]),
    "ns_lstm_set_engine": (c_int, [c_int]),
    "ns_gpt_set_comm_timing": (c_int, [P, c_int]),
    "ns_gpt_comm_times": (c_int, [P, P, P]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load libns_b200.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        import torch  # noqa: F401  (binds the shared CUDA runtime first)

        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m neuralsuite_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    lib = load()
    return [n for n in _SIGS if getattr(lib, n, None) is not None]


def check(rc: int) -> None:
    """Raise the reference-style exception for a non-OK status."""
    if rc == NS_OK:
        return
    msg = load().ns_last_error().decode(errors="replace")
    if rc == NS_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if rc == NS_ERR_OUT_OF_RANGE:
        raise IndexError(msg)
    raise NsError(rc, msg)
