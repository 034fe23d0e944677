"""NSF checkpoints against the reference's own serialisation.

The oracle here is the reference itself: oracle.ref() wraps
GPTModel::SaveWeights / LoadWeights (include/gpt.h:293-306, format in
include/serialization.h:128-287).  Files must be byte-identical to the
reference's for the same weights, load both ways, and be rejected for the
reasons the reference's tests name (test_suite.cpp:915-996): another
architecture, a truncated file, a flipped byte, a file without the header.

CPU tests use the host-side writer/reader of the library (no GPU); the GPU
tests save from and load into the device model, and resume a run from a
weights + optimizer checkpoint bit for bit.
"""
import ctypes

import numpy as np
import pytest

import oracle
from neuralsuite_b200.model import GPTConfig, init_params, nsf_load, nsf_save

CFGS = [GPTConfig(53, 16, 2, 2, 8), GPTConfig(256, 64, 4, 4, 128), GPTConfig(11, 5, 0, 1, 4)]


@pytest.fixture(scope="module")
def ref():
    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libnsref.so not built (needs the reference sources)")
    o = oracle.ref()
    o.lib.nsref_gpt_save_weights.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
    o.lib.nsref_gpt_load_weights.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
    return o


def ref_model(ref, cfg, flat=None):
    g = ref.gpt(cfg.vocab_size, cfg.block_size, cfg.n_layer, cfg.n_head, cfg.n_embd)
    if flat is not None:
        g.set_params(flat)
    return g


def weights(cfg, seed=0):
    return init_params(cfg, np.random.default_rng(seed), ln_noise=0.1)


@pytest.mark.parametrize("cfg", CFGS, ids=lambda c: f"L{c.n_layer}C{c.n_embd}")
def test_file_is_byte_identical_to_the_reference(ref, tmp_path, cfg):
    flat = weights(cfg)
    ours, theirs = tmp_path / "ours.nsf", tmp_path / "ref.nsf"
    nsf_save(cfg, flat, ours)
    assert ref.lib.nsref_gpt_save_weights(ref_model(ref, cfg, flat).h, str(theirs).encode()) == 1
    assert ours.read_bytes() == theirs.read_bytes()


@pytest.mark.parametrize("cfg", CFGS[:2], ids=lambda c: f"L{c.n_layer}C{c.n_embd}")
def test_files_load_both_ways(ref, tmp_path, cfg):
    flat = weights(cfg, 1)
    theirs = tmp_path / "ref.nsf"
    assert ref.lib.nsref_gpt_save_weights(ref_model(ref, cfg, flat).h, str(theirs).encode()) == 1
    got = nsf_load(cfg, theirs)
    assert np.array_equal(got.view(np.uint32), flat.view(np.uint32))
    ours = tmp_path / "ours.nsf"
    nsf_save(cfg, flat * 2, ours)
    g = ref_model(ref, cfg)
    assert ref.lib.nsref_gpt_load_weights(g.h, str(ours).encode()) == 1
    assert np.array_equal(g.get_params().view(np.uint32), (flat * 2).view(np.uint32))


def _corrupt(tmp_path, cfg, how):
    flat = weights(cfg, 2)
    p = tmp_path / f"{how}.nsf"
    nsf_save(cfg, flat, p)
    b = bytearray(p.read_bytes())
    if how == "truncated":
        b = b[: len(b) // 2]
    elif how == "flipped":
        b[-8] ^= 0x10  # inside the last tensor's floats, just before the checksum
    elif how == "headerless":
        b = bytearray(flat.tobytes())
    elif how == "version":
        b[8] = 2  # version field follows the 8-byte magic
    p.write_bytes(bytes(b))
    return p


@pytest.mark.parametrize("how,reason", [("truncated", "truncated"), ("flipped", "checksum"),
                                        ("headerless", "not an NSF file"), ("version", "version")])
def test_corrupt_files_are_rejected_like_the_reference(ref, tmp_path, how, reason):
    cfg = CFGS[0]
    p = _corrupt(tmp_path, cfg, how)
    with pytest.raises(ValueError, match=reason):
        nsf_load(cfg, p)
    assert ref.lib.nsref_gpt_load_weights(ref_model(ref, cfg).h, str(p).encode()) == 0


def test_other_architecture_is_rejected(ref, tmp_path):
    a, b = GPTConfig(53, 16, 2, 2, 8), GPTConfig(53, 16, 3, 2, 8)
    p = tmp_path / "a.nsf"
    nsf_save(a, weights(a), p)
    with pytest.raises(ValueError, match="n_layer is 2 in the file and 3"):
        nsf_load(b, p)
    assert ref.lib.nsref_gpt_load_weights(ref_model(ref, b).h, str(p).encode()) == 0


def test_missing_file_is_an_error(tmp_path):
    with pytest.raises(ValueError, match="cannot open"):
        nsf_load(CFGS[0], tmp_path / "nope.nsf")


# ------------------------------------------------------------------ device

@pytest.mark.gpu
def test_device_save_and_load_match_the_reference(cuda, ref, tmp_path):
    from neuralsuite_b200 import GPTModel

    cfg = GPTConfig(256, 64, 4, 4, 128)
    flat = weights(cfg, 3)
    m = GPTModel(cfg, max_batch=2)
    m.set_params(flat)
    ours, theirs = tmp_path / "dev.nsf", tmp_path / "ref.nsf"
    m.save_weights(ours)
    assert ref.lib.nsref_gpt_save_weights(ref_model(ref, cfg, flat).h, str(theirs).encode()) == 1
    assert ours.read_bytes() == theirs.read_bytes()
    m2 = GPTModel(cfg, max_batch=2)
    m2.set_params(np.zeros_like(flat))
    m2.load_weights(theirs)
    assert np.array_equal(m2.get_params().view(np.uint32), flat.view(np.uint32))
    # a rejected file leaves the device parameters as they were
    bad = _corrupt(tmp_path, cfg, "flipped")
    with pytest.raises(ValueError, match="checksum"):
        m2.load_weights(bad)
    assert np.array_equal(m2.get_params().view(np.uint32), flat.view(np.uint32))


@pytest.mark.gpu
def test_resume_from_weights_and_optimizer_is_bit_exact(cuda, tmp_path):
    """Three AdamW steps in one run against two steps, a checkpoint (weights
    + AdamW moments and step count), a fresh model loaded from it, and the
    third step: the same parameters bit for bit."""
    import torch

    from neuralsuite_b200 import GPTModel

    cfg = GPTConfig(256, 64, 4, 4, 128)
    flat = weights(cfg, 4)
    r = np.random.default_rng(5)
    tok = torch.as_tensor(r.integers(0, 256, (8, 64)).astype(np.int32), device="cuda")
    tgt = torch.as_tensor(r.integers(0, 256, 8 * 64).astype(np.int32), device="cuda")
    a = GPTModel(cfg, max_batch=8)
    a.set_params(flat)
    a.adamw_init(1e-3)
    for _ in range(3):
        a.train_step(tok, tgt)
    b = GPTModel(cfg, max_batch=8)
    b.set_params(flat)
    b.adamw_init(1e-3)
    for _ in range(2):
        b.train_step(tok, tgt)
    b.save_weights(tmp_path / "w.nsf")
    b.save_optimizer(tmp_path / "opt.nsf")
    del b
    c = GPTModel(cfg, max_batch=8)
    c.adamw_init(5e-2)  # lr, betas, eps and the step count come from the file
    c.load_weights(tmp_path / "w.nsf")
    c.load_optimizer(tmp_path / "opt.nsf")
    c.train_step(tok, tgt)
    assert np.array_equal(c.get_params().view(np.uint32), a.get_params().view(np.uint32))
    with pytest.raises(ValueError, match="arch"):
        c.load_optimizer(tmp_path / "w.nsf")  # a weights file is not an optimizer file
    d = GPTModel(cfg, max_batch=8)
    d.adamw_init(1e-3, wd=0.1)
    with pytest.raises(ValueError, match="weight_decay"):
        d.load_optimizer(tmp_path / "opt.nsf")
