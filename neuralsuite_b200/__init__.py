"""B200 (sm_100a) backend for NeuralSuite's GPT training step.

The compute lives in ``libns_b200.so`` (hand-written CUDA kernels behind the
C ABI of ``include/ns_b200.h``); this package is its Python face:

* ``kernels`` -- one wrapper per kernel entry point (MatMul, attention,
  LayerNorm, GELU, cross-entropy, embedding, AdamW), for tests and tools;
* ``model`` -- the device GPTModel + CrossEntropyLoss + AdamW step, its NSF
  checkpoints, the KV-cache ``Decoder``, the diffusion ``UNet`` step and the
  NCCL communicator used for data parallel training.
"""
from .model import (Comm, Decoder, GPTConfig, GPTModel, UNet, init_params,  # noqa: F401
                    nsf_load, nsf_save, param_shapes, plan_buckets)

__all__ = ["Comm", "Decoder", "GPTConfig", "GPTModel", "UNet", "init_params", "nsf_load",
           "nsf_save", "param_shapes", "plan_buckets"]
