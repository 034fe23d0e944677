"""KV-cache decoding against the reference's GPTModel::ForwardWithKVCache
(include/gpt.h:159-190; the cache of include/layers/attention.h:481-546),
driven like generate_llm.cpp:146-160: the prompt token by token at
positions 0..n-1, then generation re-feeding the last token at position n-1
before each new one (the reference's loop does exactly that).

Every step's logits are held to the north-star tolerance against the
compiled reference, with float64 adjudication (oracle/fp64.gpt_decode) of
the elements that miss.
"""
import numpy as np
import pytest
import torch

import oracle
from neuralsuite_b200 import Decoder, GPTConfig, GPTModel, init_params
from oracle import fp64
from tests._util import close_report

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libnsref.so not built (needs the reference sources)")
    o = oracle.ref()
    o.set_threads(8)
    return o


def generate_steps(prompt, extra):
    """(token, pos) sequence of generate_llm.cpp's cached loop."""
    steps = [(t, p) for p, t in enumerate(prompt)]
    toks = list(prompt)
    for t in extra:
        steps.append((toks[-1], len(toks) - 1))
        toks.append(t)
    return steps


def ref_decode(ref, cfg, flat, steps):
    g = ref.gpt(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd)
    g.set_params(flat)
    g.clear_kv()
    return np.array([g.decode(t, p) for t, p in steps])


def check_steps(tag, got, want, flat, cfg, steps):
    ok, info = close_report(got, want)
    if not ok:
        f = fp64.gpt_decode(flat, steps, cfg.vocab_size, cfg.block_size, cfg.n_layer,
                            cfg.n_head, cfg.n_embd)
        ok, info = close_report(got, want, f)
    assert ok, (tag, info)
    return info


@pytest.mark.parametrize("cfg", [GPTConfig(256, 64, 4, 4, 128), GPTConfig(53, 32, 2, 2, 8),
                                 GPTConfig(256, 48, 2, 1, 96)],
                         ids=["c1", "tiny", "head96"])
def test_token_by_token_matches_reference(cuda, ref, cfg):
    r = np.random.default_rng(cfg.n_embd + cfg.n_layer)
    flat = init_params(cfg, r, ln_noise=0.1)
    prompt = r.integers(0, cfg.vocab_size, 9).tolist()
    steps = generate_steps(prompt, r.integers(0, cfg.vocab_size, 6).tolist())
    want = ref_decode(ref, cfg, flat, steps)
    m = GPTModel(cfg, max_batch=1)
    m.set_params(flat)
    dec = Decoder(m, max_batch=1)
    got = np.array([dec.step([t], p).cpu().numpy()[0] for t, p in steps])
    dec.check()
    assert len(dec) == len(steps)
    check_steps("decode", got, want, flat, cfg, steps)


def test_batched_sequences_match_the_reference_one_by_one(cuda, ref):
    """Three sequences in lockstep; each row against its own reference run."""
    cfg = GPTConfig(256, 64, 4, 4, 128)
    r = np.random.default_rng(3)
    flat = init_params(cfg, r, ln_noise=0.1)
    toks = r.integers(0, 256, (3, 14))
    m = GPTModel(cfg, max_batch=3)
    m.set_params(flat)
    dec = Decoder(m, max_batch=3)
    got = np.stack([dec.step(toks[:, p], p).cpu().numpy() for p in range(14)], 1)  # [3, 14, V]
    for b in range(3):
        steps = [(int(t), p) for p, t in enumerate(toks[b])]
        check_steps(f"seq {b}", got[b], ref_decode(ref, cfg, flat, steps), flat, cfg, steps)


def test_prefill_equals_decoding_the_prompt(cuda, ref):
    """The batched prefill (training forward + cache fill) leaves the cache
    that decoding the prompt token by token leaves: its last logits and the
    following decode steps match the reference's token-by-token run."""
    cfg = GPTConfig(256, 64, 4, 4, 128)
    r = np.random.default_rng(4)
    flat = init_params(cfg, r, ln_noise=0.1)
    B, T = 2, 20
    prompt = r.integers(0, 256, (B, T))
    nxt = r.integers(0, 256, (B, 5))
    m = GPTModel(cfg, max_batch=B)
    m.set_params(flat)
    dec = Decoder(m, max_batch=B)
    last = dec.prefill(prompt).cpu().numpy()
    assert len(dec) == T
    rows = [last] + [dec.step(nxt[:, i], T + i).cpu().numpy() for i in range(5)]
    got = np.stack(rows, 1)  # [B, 6, V]
    for b in range(B):
        steps = [(int(t), p) for p, t in enumerate(prompt[b])] + \
                [(int(nxt[b, i]), T + i) for i in range(5)]
        want = ref_decode(ref, cfg, flat, steps)[T - 1:]
        f64 = fp64.gpt_decode(flat, steps, 256, 64, 4, 4, 128)[T - 1:]
        ok, info = close_report(got[b], want, f64)
        assert ok, (b, info)


@pytest.mark.slow
def test_gpt12x768_prefill_and_decode(cuda, ref):
    """The 12-layer/768 model: a 32-token prompt by prefill, then 4 steps."""
    cfg = GPTConfig(256, 1024, 12, 12, 768)
    r = np.random.default_rng(5)
    flat = init_params(cfg, r)
    prompt = r.integers(0, 256, 32)
    nxt = r.integers(0, 256, 4)
    m = GPTModel(cfg, max_batch=1)
    m.set_params(flat)
    dec = Decoder(m, max_batch=1)
    rows = [dec.prefill(prompt[None]).cpu().numpy()[0]]
    rows += [dec.step([int(nxt[i])], 32 + i).cpu().numpy()[0] for i in range(4)]
    steps = [(int(t), p) for p, t in enumerate(prompt)] + [(int(nxt[i]), 32 + i) for i in range(4)]
    want = ref_decode(ref, cfg, flat, steps)[31:]
    check_steps("12x768", np.array(rows), want, flat, cfg, steps)


def test_decoder_errors(cuda):
    cfg = GPTConfig(16, 4, 1, 2, 8)
    m = GPTModel(cfg, max_batch=2)
    m.set_params(init_params(cfg, np.random.default_rng(0)))
    dec = Decoder(m, max_batch=2)
    with pytest.raises(IndexError):
        dec.step([0], 4)  # position beyond block_size
    with pytest.raises(IndexError):
        dec.step([99], 0)  # host-side token check (std::out_of_range)
    dec.step(torch.tensor([99], dtype=torch.int32, device="cuda"), 0)  # device token: flagged
    with pytest.raises(IndexError):
        dec.check()
    dec.clear()
    for p in range(4):
        dec.step([1, 2], p)
    with pytest.raises(IndexError):
        dec.step([1, 2], 3)  # the cache holds block_size positions
    with pytest.raises(ValueError):
        dec.step([1], 0)  # another batch size while the cache holds two sequences
    dec.clear()
    dec.step([1], 0)
    assert len(dec) == 1
