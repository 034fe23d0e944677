"""CPU checks of the C ABI's error behaviour: invalid arguments come back as
the status codes of the reference's exception types, with a message, before
any device work is issued.

Every call below is rejected by the library's own argument checks before it
touches a pointer or launches a kernel, so these tests need no GPU and are
safe where one is present.  The pointers passed are never dereferenced.
"""
import ctypes

import pytest

NS_OK, NS_ERR_INVALID_ARGUMENT, NS_ERR_OUT_OF_RANGE = 0, 1, 2

FAKE = ctypes.c_void_p(0x10000)  # 16-byte aligned, never dereferenced (rejected first)
FAKE_MISALIGNED = ctypes.c_void_p(0x10004)


@pytest.fixture(scope="module")
def lib():
    from neuralsuite_b200 import _lib

    return _lib.load()


def _err(lib, rc, code, text):
    assert rc == code, (rc, lib.ns_last_error())
    assert text in lib.ns_last_error().decode(), lib.ns_last_error()


def test_gpt_create_rejects_n_embd_not_divisible_by_n_head(lib):
    """MultiHeadAttention's constructor check (include/layers/attention.h)."""
    from neuralsuite_b200 import _lib

    cfg = _lib.ns_gpt_config(256, 64, 2, 4, 130, 1)
    h = ctypes.c_void_p()
    _err(lib, lib.ns_gpt_create(ctypes.byref(cfg), ctypes.byref(h)), NS_ERR_INVALID_ARGUMENT,
         "n_head")
    assert not h.value


@pytest.mark.parametrize("field", ["vocab", "block", "embd", "batch"])
def test_gpt_create_rejects_non_positive_sizes(lib, field):
    from neuralsuite_b200 import _lib

    v = dict(vocab=256, block=64, embd=128, batch=1)
    v[field] = 0
    cfg = _lib.ns_gpt_config(v["vocab"], v["block"], 2, 4, v["embd"], v["batch"])
    h = ctypes.c_void_p()
    rc = lib.ns_gpt_create(ctypes.byref(cfg), ctypes.byref(h))
    assert rc == NS_ERR_INVALID_ARGUMENT, lib.ns_last_error()
    assert not h.value


def test_gpt_create_rejects_null(lib):
    h = ctypes.c_void_p()
    _err(lib, lib.ns_gpt_create(None, ctypes.byref(h)), NS_ERR_INVALID_ARGUMENT, "NULL")


def _gemm(lib, M=4, N=4, K=4, lda=4, ldb=4, ldc=4, beta=0.0, epi=0, bias=None):
    return lib.ns_gemm(M, N, K, FAKE, lda, 0, FAKE, ldb, 0, FAKE, ldc, beta, epi, bias, None,
                       None, None, 0, None)


def test_gemm_argument_checks(lib):
    _err(lib, _gemm(lib, M=-1), NS_ERR_INVALID_ARGUMENT, "negative dimension")
    _err(lib, _gemm(lib, beta=0.5), NS_ERR_INVALID_ARGUMENT, "beta")
    _err(lib, _gemm(lib, ldc=3), NS_ERR_INVALID_ARGUMENT, "ldc")
    _err(lib, _gemm(lib, lda=3), NS_ERR_INVALID_ARGUMENT, "leading dimension")
    _err(lib, _gemm(lib, epi=99), NS_ERR_INVALID_ARGUMENT, "epilogue")
    _err(lib, _gemm(lib, epi=1), NS_ERR_INVALID_ARGUMENT, "bias")  # NS_EPI_BIAS without bias


def test_gemm_with_an_empty_output_is_a_no_op(lib):
    assert _gemm(lib, M=0) == NS_OK
    assert _gemm(lib, N=0, ldc=0, ldb=0) == NS_OK


def test_layernorm_backward_checks(lib):
    rc = lib.ns_layernorm_bwd(FAKE, FAKE, FAKE, FAKE, FAKE, None, FAKE, FAKE, FAKE, -1, 16, None,
                              0, None)
    _err(lib, rc, NS_ERR_INVALID_ARGUMENT, "rows")
    rc = lib.ns_layernorm_bwd(FAKE, FAKE, FAKE, FAKE, FAKE, None, FAKE, FAKE, FAKE, 8, 16, None,
                              0, None)
    _err(lib, rc, NS_ERR_INVALID_ARGUMENT, "workspace")


def test_embedding_rejects_a_sequence_longer_than_block_size(lib):
    """The reference throws std::out_of_range (include/gpt.h Forward)."""
    rc = lib.ns_embedding_fwd(FAKE, 1, 65, FAKE, 256, FAKE, 64, 128, FAKE, FAKE, None)
    _err(lib, rc, NS_ERR_OUT_OF_RANGE, "block_size")


def _adamw(lib, offsets, decay, ptr=FAKE, n_total=None):
    n = len(decay)
    offs = (ctypes.c_int64 * (n + 1))(*offsets)
    dec = (ctypes.c_float * max(1, n))(*decay)
    total = offsets[-1] if n_total is None else n_total
    return lib.ns_adamw_flat(ptr, FAKE, FAKE, FAKE, total, ctypes.cast(offs, ctypes.c_void_p),
                             ctypes.cast(dec, ctypes.c_void_p), n, 1e-3, 0.9, 0.95, 1e-8, 0.1,
                             0.05, None)


def test_adamw_checks_the_segment_table_before_launching(lib):
    _err(lib, _adamw(lib, [0, 8, 4, 12], [0.0, 0.1, 0.0]), NS_ERR_INVALID_ARGUMENT, "ascending")
    _err(lib, _adamw(lib, [0, 8, 16], [0.0, 0.1], n_total=12), NS_ERR_INVALID_ARGUMENT,
         "exceed")
    _err(lib, _adamw(lib, [0, 8], [0.0], ptr=FAKE_MISALIGNED), NS_ERR_INVALID_ARGUMENT,
         "aligned")


def test_attention_backward_checks(lib):
    def bwd(B, T, H, D, ws=None):
        return lib.ns_attn_bwd(FAKE, FAKE, FAKE, FAKE, B, T, H, D, FAKE, ws, 0, None)

    _err(lib, bwd(1, 4, 1, 256), NS_ERR_INVALID_ARGUMENT, "head_dim")
    _err(lib, bwd(1, 4, 0, 64), NS_ERR_INVALID_ARGUMENT, "bad shape")
    _err(lib, bwd(1, 4, 1, 64), NS_ERR_INVALID_ARGUMENT, "workspace")
    assert bwd(0, 4, 1, 64) == NS_OK  # an empty batch is no work


def test_cross_entropy_checks(lib):
    def ce(rows, classes, denom, ws=None):
        return lib.ns_cross_entropy(FAKE, FAKE, rows, classes, denom, FAKE, FAKE, FAKE, ws, 0,
                                    None)

    _err(lib, ce(0, 256, 1.0), NS_ERR_INVALID_ARGUMENT, "positive")
    _err(lib, ce(8, 0, 1.0), NS_ERR_INVALID_ARGUMENT, "positive")
    _err(lib, ce(8, 256, 0.0), NS_ERR_INVALID_ARGUMENT, "denom")
    _err(lib, ce(8, 256, 8.0), NS_ERR_INVALID_ARGUMENT, "workspace")


def test_bias_gradient_split_checks(lib):
    def bgs(M, N, dy=FAKE, ws=None):
        return lib.ns_bias_grad_split(dy, M, N, FAKE, FAKE, ws, 0, None)

    _err(lib, bgs(8, 6), NS_ERR_INVALID_ARGUMENT, "multiple of 4")
    _err(lib, bgs(8, 8, dy=FAKE_MISALIGNED), NS_ERR_INVALID_ARGUMENT, "aligned")
    _err(lib, bgs(8, 8), NS_ERR_INVALID_ARGUMENT, "workspace")


def test_layernorm_forward_checks(lib):
    _err(lib, lib.ns_layernorm_fwd(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 8, 0, 1e-5, None),
         NS_ERR_INVALID_ARGUMENT, "dim")
    # a residual to add needs the bias and the buffer the sum goes to
    rc = lib.ns_layernorm_fwd_ex(FAKE, None, FAKE, FAKE, FAKE, FAKE, FAKE, None, FAKE, FAKE, 8,
                                 16, 1e-5, None)
    _err(lib, rc, NS_ERR_INVALID_ARGUMENT, "resid")


def test_pointwise_and_split_checks(lib):
    _err(lib, lib.ns_gelu_fwd_lo(FAKE, FAKE, FAKE_MISALIGNED, 16, None), NS_ERR_INVALID_ARGUMENT,
         "aligned")
    _err(lib, lib.ns_gelu_fwd(FAKE, FAKE, -1, None), NS_ERR_INVALID_ARGUMENT, "n < 0")
    _err(lib, lib.ns_split_lo(FAKE, 4, 8, 4, FAKE, None), NS_ERR_INVALID_ARGUMENT, "bad shape")
    assert lib.ns_split_lo(FAKE, 0, 8, 8, FAKE, None) == NS_OK


@pytest.mark.parametrize("call", ["forward", "loss_backward", "backward", "adamw_init",
                                  "adamw_set_lr", "adamw_step", "clip_gradients", "train_step",
                                  "set_comm", "set_comm_timing", "comm_times"])
def test_model_entry_points_reject_a_null_handle(lib, call):
    args = {
        "forward": (None, FAKE, 1, 1, None),
        "loss_backward": (None, FAKE, None),
        "backward": (None, None),
        "adamw_init": (None, 1e-3, 0.9, 0.95, 1e-8, 0.01),
        "adamw_set_lr": (None, 1e-3),
        "adamw_step": (None, None),
        "clip_gradients": (None, 1.0, None),
        "train_step": (None, FAKE, FAKE, 1, 1, 0.0, None, None),
        "set_comm": (None, None, 1, 0),
        "set_comm_timing": (None, 1),
        "comm_times": (None, FAKE, FAKE),
    }[call]
    _err(lib, getattr(lib, "ns_gpt_" + call)(*args), NS_ERR_INVALID_ARGUMENT, "NULL model")


def test_model_getters_tolerate_a_null_handle(lib):
    assert lib.ns_gpt_num_tensors(None) == 0
    assert lib.ns_gpt_num_params(None) == 0
    assert lib.ns_gpt_tensor_numel(None, 0) == 0
    assert not lib.ns_gpt_params(None)


def test_noalloc_cross_entropy_rejects_rows_beyond_its_static_scratch(lib):
    """ns_cross_entropy_noalloc keeps its per-row scratch in a fixed device
    array of NS_CE_NOALLOC_MAX_ROWS floats; a larger call is refused before
    any device work, so this runs without a GPU."""
    rows = 65536 + 1
    rc = lib.ns_cross_entropy_noalloc(FAKE, FAKE, rows, 4, float(rows), FAKE, FAKE, FAKE, None)
    _err(lib, rc, NS_ERR_INVALID_ARGUMENT, "NS_CE_NOALLOC_MAX_ROWS")


def test_conv2d_rejects_bad_parameters(lib):
    """Conv2D's constructor and Forward checks (include/layers/conv2d.h:203-224)
    as std::invalid_argument, before any device work."""
    assert lib.ns_conv2d_workspace_size(1, 3, 2, 2, 4, 5, 1, 0) == 0  # kernel larger than input
    _err(lib, lib.ns_conv2d_fwd(FAKE, 1, 3, 2, 2, FAKE, FAKE, 4, 5, 1, 0, FAKE, None, 0, None),
         NS_ERR_INVALID_ARGUMENT, "does not fit")
    _err(lib, lib.ns_conv2d_fwd(FAKE, 1, 3, 8, 8, FAKE, FAKE, 4, 3, 0, 1, FAKE, None, 0, None),
         NS_ERR_INVALID_ARGUMENT, "bad convolution")
    _err(lib, lib.ns_conv2d_fwd(FAKE, 1, 3, 8, 8, FAKE, FAKE, 4, 3, 1, 1, FAKE, FAKE, 0, None),
         NS_ERR_INVALID_ARGUMENT, "workspace")


def test_lstm_engine_checks(lib):
    _err(lib, lib.ns_lstm_set_engine(2), NS_ERR_INVALID_ARGUMENT, "engine")
    assert lib.ns_lstm_set_engine(0) == NS_OK


def test_gemm_engine_checks(lib):
    """Engines 0-11 are accepted (10 / 11 force the CTA-pair kernel's fixed or
    counter-driven work order); anything else is rejected with a message."""
    for bad in (-1, 12):
        _err(lib, lib.ns_gemm_set_engine(bad), NS_ERR_INVALID_ARGUMENT, "engine")
    try:
        for good in (10, 11, 0):
            assert lib.ns_gemm_set_engine(good) == NS_OK
    finally:
        assert lib.ns_gemm_set_engine(0) == NS_OK
