"""Model-level parity of the device GPT training step against the reference.

Tolerance (north star): loss, logits and every gradient within
|x - ref| <= 1e-5 + 1e-4*|ref| of the fp32 CPU reference, misses adjudicated
against the float64 restatement (tests/_util.close_report).  Token handling
is bit-exact (checked at kernel level in test_gpu_kernels.py).
"""
import os

import numpy as np
import pytest
import torch

from neuralsuite_b200 import GPTConfig, GPTModel, param_shapes
from oracle import fp64
from tests._util import close_report, gpt_init, rng

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def check_step(tag, loss, logits, grads, ref_loss, ref_logits, ref_grads, f64):
    l64, lg64, g64 = f64
    ok, info = close_report(np.array([loss]), np.array([ref_loss]), np.array([l64]))
    assert ok, (tag, "loss", loss, ref_loss, info)
    ok, info = close_report(logits, ref_logits, lg64)
    assert ok, (tag, "logits", info)
    ok, info = close_report(grads, ref_grads, g64)
    assert ok, (tag, "grads", info)


def check_params_after_adam(tag, got, ref, lr, steps):
    """After AdamW the update of a parameter whose gradient is at rounding
    level can take either sign (m/sqrt(v) ~ +-1), so the bound is: 99.9% of
    parameters within the step tolerance and all within 2*lr*steps."""
    err = np.abs(got.astype(np.float64) - ref.astype(np.float64))
    tight = err <= 1e-5 + 1e-4 * np.abs(ref)
    assert tight.mean() >= 0.999, (tag, float(tight.mean()), float(err.max()))
    assert err.max() <= 2 * lr * steps + 1e-6, (tag, float(err.max()))


@pytest.mark.parametrize("name", ["gpt_tiny", "gpt_small"])
def test_golden_steps(cuda, name):
    """The reference's own numbers (tests/golden, produced by the reference
    from its sources): loss, logits, all gradients, then AdamW steps."""
    f = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    V, block, L, H, C, B, T, steps = (int(v) for v in f["cfg"])
    m = GPTModel(GPTConfig(V, block, L, H, C), max_batch=B)
    assert m.n_tensors == 2 + 12 * L + 2
    m.set_params(f["params0"])
    m.adamw_init(3e-4)
    f64 = fp64.gpt_fwd_bwd(f["params0"], f["idx"], f["targets"], V, block, L, H, C)
    losses = []
    for s in range(steps):
        loss, logits = m.fwd_bwd(f["idx"], f["targets"])
        losses.append(loss)
        if s == 0:
            check_step(name, loss, logits, m.get_grads(), float(f["loss0"][0]), f["logits0"],
                       f["grads0"], f64)
        m.adamw_step()
    assert np.allclose(losses, f["losses"], rtol=1e-4, atol=1e-5), (losses, f["losses"])
    check_params_after_adam(name, m.get_params(), f["params_final"], 3e-4, steps)


def c1_inputs(seed=1234, B=8, T=64, V=256):
    r = rng(seed)
    cfg = GPTConfig(vocab_size=V, block_size=64, n_layer=4, n_head=4, n_embd=128)
    flat = gpt_init(param_shapes(cfg), r, ln_noise=0.05)
    idx = r.integers(0, V, (B, T)).astype(np.float32)
    tgt = r.integers(0, V, B * T).astype(np.float32)
    return cfg, flat, idx, tgt


def test_config1_step_vs_oracle(cuda, port):
    """4 layers, n_embd 128, 4 heads, T=64, B=8, vocab 256: forward, CE,
    backward and three AdamW(lr=3e-4) steps against the C oracle (bit-identical
    to the reference) on the same seeded weights and byte tokens."""
    cfg, flat, idx, tgt = c1_inputs()
    m = GPTModel(cfg, max_batch=8)
    m.set_params(flat)
    o = port.gpt(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd)
    o.set_params(flat)
    f64 = fp64.gpt_fwd_bwd(flat, idx, tgt, cfg.vocab_size, cfg.block_size, cfg.n_layer,
                           cfg.n_head, cfg.n_embd)
    loss, logits = m.fwd_bwd(idx, tgt)
    rl, rlog = o.fwd_bwd(idx, tgt)
    check_step("c1", loss, logits, m.get_grads(), rl, rlog, o.get_grads(), f64)
    m.adamw_init(3e-4)
    o.adamw_init(3e-4)
    m.adamw_step()
    o.adamw_step()
    for _ in range(2):
        m.fwd_bwd(idx, tgt)
        o.fwd_bwd(idx, tgt)
        m.adamw_step()
        o.adamw_step()
    check_params_after_adam("c1", m.get_params(), o.get_params(), 3e-4, 3)


def test_train_step_matches_parts_and_learns(cuda):
    cfg, flat, idx, tgt = c1_inputs(seed=7)
    m = GPTModel(cfg, max_batch=8)
    m.set_params(flat)
    m.adamw_init(3e-3)
    tok = torch.as_tensor(idx.astype(np.int32), device="cuda")
    tg = torch.as_tensor(tgt.astype(np.int32), device="cuda")
    losses = [m.train_step(tok, tg) for _ in range(8)]
    assert all(np.isfinite(losses))
    assert losses[-1] < losses[0] - 0.05, losses
    m2 = GPTModel(cfg, max_batch=8)
    m2.set_params(flat)
    l0, _ = m2.fwd_bwd(idx, tgt)
    assert abs(l0 - losses[0]) <= 1e-6 * abs(l0), (l0, losses[0])


@pytest.mark.parametrize("max_norm", [0.01, 1e6])
def test_clip_gradients(cuda, port, max_norm):
    """ClipGradients(params, max_norm) of train_llm.cpp:112-129 on device
    against the oracle's restatement (serial float sum of squares, then the
    in-place scale by max_norm / norm when norm > max_norm) after the same
    forward/backward; 1e6 leaves the gradients untouched."""
    cfg, flat, idx, tgt = c1_inputs(seed=3)
    m = GPTModel(cfg, max_batch=8)
    m.set_params(flat)
    m.fwd_bwd(idx, tgt)
    o = port.gpt(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd)
    o.set_params(flat)
    o.fwd_bwd(idx, tgt)
    norm_ref = o.clip_gradients(max_norm)
    _, _, g64 = fp64.gpt_fwd_bwd(flat, idx, tgt, cfg.vocab_size, cfg.block_size, cfg.n_layer,
                                 cfg.n_head, cfg.n_embd)
    norm64 = float(np.sqrt((g64 * g64).sum()))
    # The reference's serial float sum of 800K squares drifts from the exact
    # norm (6.6e-4 relative here); the device's tree sum stays near float64.
    # Elements that miss the fp32 reference by more than the tolerance pass
    # only where the device is as close to the float64 result as the
    # reference is (close_report's adjudication).
    assert abs(norm_ref - norm64) <= 1e-2 * norm64, (norm_ref, norm64)
    m.clip_gradients(max_norm)
    want64 = g64 * (max_norm / norm64) if norm64 > max_norm else g64
    ok, info = close_report(m.get_grads(), o.get_grads(), want64)
    assert ok, info


def test_step_is_deterministic(cuda):
    cfg, flat, idx, tgt = c1_inputs(seed=11)
    m = GPTModel(cfg, max_batch=8)
    m.set_params(flat)
    l1, lg1 = m.fwd_bwd(idx, tgt)
    g1 = m.get_grads()
    l2, lg2 = m.fwd_bwd(idx, tgt)
    g2 = m.get_grads()
    assert l1 == l2
    assert np.array_equal(lg1.view(np.uint32), lg2.view(np.uint32))
    assert np.array_equal(g1.view(np.uint32), g2.view(np.uint32))


def test_reference_errors(cuda):
    """Errors surface as the reference's exceptions (test_suite.cpp:334-362)."""
    cfg = GPTConfig(vocab_size=10, block_size=4, n_layer=1, n_head=2, n_embd=8)
    m = GPTModel(cfg, max_batch=2)
    with pytest.raises(IndexError):  # std::out_of_range, embedding.h:45-49
        m.forward(np.array([[0, 999]], np.float32))
    with pytest.raises(IndexError):  # position beyond block_size
        m.forward(np.zeros((1, 5), np.float32))
    with pytest.raises(ValueError):  # attention.h:341-345
        GPTModel(GPTConfig(vocab_size=16, block_size=8, n_layer=1, n_head=4, n_embd=130), 1)
    with pytest.raises(ValueError):
        m.set_params(np.zeros(3, np.float32))


@pytest.mark.slow
def test_config4_step_properties(cuda):
    """12 layers, n_embd 768, 12 heads, T=1024, B=8: at N(0, 0.02) init each
    logit is a sum of 768 products of a unit-variance LayerNorm output with
    N(0, 0.02) wte entries, i.e. ~N(0, s2) with s2 = 768 * 0.02^2, so the
    expected loss is ln(256) + s2/2; gradients are finite and the step is
    bit-reproducible; a small AdamW step on the batch lowers its loss (the
    first Adam step moves every parameter by ~lr, so at lr 3e-4 over 86M
    parameters the second-order term can dominate; 3e-5 keeps it first-order)."""
    cfg = GPTConfig(vocab_size=256, block_size=1024, n_layer=12, n_head=12, n_embd=768)
    r = rng(99)
    flat = gpt_init(param_shapes(cfg), r)
    B, T = 8, 1024
    tok = torch.as_tensor(r.integers(0, 256, (B, T)).astype(np.int32), device="cuda")
    tgt = torch.as_tensor(r.integers(0, 256, B * T).astype(np.int32), device="cuda")
    m = GPTModel(cfg, max_batch=B)
    m.set_params(flat)
    assert m.n_params == 86_039_040 and m.n_tensors == 148
    m.forward(tok)
    loss = float(m.loss_backward(tgt).item())
    expected = np.log(256.0) + 768 * 0.02 ** 2 / 2
    assert abs(loss - expected) < 0.02, (loss, expected)
    m.backward()
    g1 = m.grads().clone()
    assert torch.isfinite(g1).all()
    m.forward(tok)
    m.loss_backward(tgt)
    m.backward()
    assert torch.equal(g1, m.grads())
    m.adamw_init(3e-5)
    m.adamw_step()
    m.forward(tok)
    loss2 = float(m.loss_backward(tgt).item())
    assert loss2 < loss, (loss, loss2)
