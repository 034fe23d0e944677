"""CPU checks of the C ABI: the library builds for sm_100a, loads, and exports
every entry point declared in include/ns_b200.h (no kernel is launched)."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "ns_b200.h")).read()
    return sorted(set(re.findall(r"^NS_API [^(]*?\b(ns_\w+)\(", text, flags=re.M)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("ns_gemm", "ns_attn_fwd", "ns_attn_bwd", "ns_layernorm_fwd", "ns_layernorm_bwd",
              "ns_embedding_fwd", "ns_embedding_bwd", "ns_cross_entropy", "ns_adamw_flat",
              "ns_gpt_create", "ns_gpt_train_step", "ns_comm_init"):
        assert s in syms, s


def test_library_exports_every_declared_symbol():
    from neuralsuite_b200 import _lib

    lib = _lib.load()
    missing = [s for s in declared_symbols() if getattr(lib, s, None) is None]
    assert not missing, missing
    assert lib.ns_version() >= 1


def test_binding_signatures_cover_header():
    from neuralsuite_b200 import _lib

    assert set(declared_symbols()) <= set(_lib._SIGS), set(declared_symbols()) - set(_lib._SIGS)


def test_attention_forward_rejects_a_missing_workspace():
    """Argument checks run before any device work: head size 64 needs the
    K/V lo-part workspace, head size 16 needs none."""
    from neuralsuite_b200 import _lib

    lib = _lib.load()
    assert lib.ns_attn_fwd_workspace_size(2, 128, 4, 64) == 2 * 128 * 2 * 4 * 64 * 4
    assert lib.ns_attn_fwd_workspace_size(2, 128, 4, 16) == 0
    rc = lib.ns_attn_fwd(None, 1, 4, 1, 64, None, None, None, 0, None)
    assert rc == 1  # NS_ERR_INVALID_ARGUMENT
    assert b"workspace" in lib.ns_last_error()
