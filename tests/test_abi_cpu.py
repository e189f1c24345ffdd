"""The C-ABI library, checked without a GPU: it loads, exports exactly what
include/g4.h declares, and its host-side argument checks behave (no kernel runs)."""

import ctypes

import pytest

import g4b200


def test_library_loads_and_reports_version():
    assert g4b200.LIB.g4_version().startswith(b"g4b200")


def test_every_header_symbol_is_exported():
    declared = g4b200.header_symbols()
    assert len(declared) >= 20
    assert g4b200.exported_symbols() == declared


def test_reference_entry_points_are_declared():
    # one C entry point per #[device] text op of src/ops.rs
    ops = ["embed_token", "copy_hidden_state", "sliding_project_qkv", "full_project_qkv", "sliding_attention",
           "sliding_attention_output", "full_attention_first_page", "full_attention_page",
           "full_attention_output", "decoder_feedforward", "final_norm_and_logits"]
    declared = set(g4b200.header_symbols())
    for op in ops:
        assert f"g4_{op}" in declared


def test_null_context_is_rejected():
    null = ctypes.c_void_p(0)
    assert g4b200.LIB.g4_decoder_feedforward(null, *([None] * 13)) == 1
    assert g4b200.LIB.g4_sliding_attention(null, None, None, None, None, None) == 1
    assert g4b200.LIB.g4_ctx_set_wait_budget(null, 5) == 1
    assert g4b200.LIB.g4_ctx_last_error(null) == b"null context"


def test_context_creation_fails_cleanly_without_a_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    assert g4b200.LIB.g4_ctx_create(0, ctypes.byref(h)) == 2  # G4_ERR_CUDA
    assert not h.value
    with pytest.raises(g4b200.G4Error):
        g4b200.Context(0)
