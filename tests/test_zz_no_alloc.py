"""g4_decoder_feedforward_noalloc: decoder_feedforward for hosts that forbid this library
to allocate device memory (its scratch is one fixed array per GPU in the library image).

Named to be collected last, so that it also runs after every other test has used the
context entry points; it must pass as well when run alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

import g4b200 as g4
from g4formats import quant
from oracle import cases, ops

MLP_ARGS = ("residual", "pre_ff_rms_weight", "up_weight_packed", "gate_weight_packed", "down_weight_packed",
            "up_weight_scale", "gate_weight_scale", "down_weight_scale", "up_global_scale", "gate_global_scale",
            "down_global_scale", "post_ff_rms_weight", "layer_scalar")
# the decoder_feedforward tolerance of the parity tests (oracle ATOL, plus a rel-L2 bound)
MLP_ATOL, MLP_REL_L2 = 0.02, 1e-2


def _raw(n: int, ptrs=None) -> int:
    f = g4.LIB.g4_decoder_feedforward_noalloc
    return f(None, ctypes.c_uint32(n), *(ptrs or [None] * 13))


# ----------------------------------------------------------------------- host-side checks
# Sizes and pointers are checked before any CUDA call, so these run without a GPU.
def test_rejects_intermediate_beyond_scratch_limit():
    assert g4.NOALLOC_MAX_INTERMEDIATE == 15360
    assert _raw(g4.NOALLOC_MAX_INTERMEDIATE + 128) == 6  # G4_ERR_TOO_LARGE
    assert _raw(1 << 31) == 6
    assert g4.STATUS[6] == "TOO_LARGE"


def test_rejects_unsupported_shapes_and_null_pointers():
    assert _raw(11520) == 5  # 3 K-segments per down row: not built
    assert _raw(200) == 5    # not a multiple of 128
    assert _raw(5120) == 5   # between 3840 and 7680: not a built down-phase geometry
    assert _raw(3968) == 5
    assert _raw(0) == 1
    assert _raw(15360) == 1  # null pointers


# ------------------------------------------------------------------------------ on a GPU
def _oracle(m: dict) -> np.ndarray:
    a = {k: v.cpu() for k, v in m.items()}
    f = lambda t: t.float().numpy().reshape(-1)  # noqa: E731
    n = a["gate_weight_packed"].numel() * 2 // ops.H
    return ops.decoder_feedforward(
        f(a["residual"]), f(a["pre_ff_rms_weight"]), f(a["post_ff_rms_weight"]),
        a["up_weight_packed"].numpy().reshape(n, ops.H // 2), a["gate_weight_packed"].numpy().reshape(n, ops.H // 2),
        a["down_weight_packed"].numpy().reshape(ops.H, n // 2), a["up_weight_scale"].numpy().reshape(n, -1),
        a["gate_weight_scale"].numpy().reshape(n, -1), a["down_weight_scale"].numpy().reshape(ops.H, -1),
        np.float32(a["up_global_scale"][0]), np.float32(a["gate_global_scale"][0]),
        np.float32(a["down_global_scale"][0]), f(a["layer_scalar"])[0])


def _check(want, got, label):
    r = cases.compare(np.asarray(want, np.float32), got.float().cpu().numpy(), MLP_ATOL)
    print(label, r)
    assert r["max_abs"] <= MLP_ATOL and r["rel_l2"] <= MLP_REL_L2, (label, r)


@pytest.mark.gpu
def test_noalloc_matches_context_entry_point_on_two_calls():
    """Two calls in a row on each path (the second starts from the first's output), so
    the shared array's leftover contents from call 1 must not disturb call 2."""
    ctx = g4.Context(0)
    m = {k: v.cuda() for k, v in quant.mlp_config1(seed=11, device="cpu").items()}
    res_ctx = m["residual"].clone()
    res_na = m["residual"].clone()
    for call in range(2):
        g4.decoder_feedforward(ctx, res_ctx, *[m[k] for k in MLP_ARGS[1:]])
        g4.decoder_feedforward_noalloc(res_na, *[m[k] for k in MLP_ARGS[1:]])
        torch.cuda.synchronize()
        _check(res_ctx.float().cpu().numpy(), res_na, f"call {call}")
        assert not torch.equal(res_na, m["residual"])  # the residual really was updated
    assert ctx.poll() == 0
    ctx.close()


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [7680, 1920])
def test_noalloc_smaller_intermediate_vs_oracle(rows):
    m = quant.mlp_config1(seed=3, device="cpu", rows=rows)
    want = _oracle(m)
    d = {k: v.cuda() for k, v in m.items()}
    g4.decoder_feedforward_noalloc(*[d[k] for k in MLP_ARGS])
    torch.cuda.synchronize()
    _check(want, d["residual"], f"rows {rows}")


@pytest.mark.gpu
def test_noalloc_oversize_raises_before_launch():
    rows = g4.NOALLOC_MAX_INTERMEDIATE + 128
    d = {k: v.cuda() for k, v in quant.mlp_config1(seed=5, device="cpu", rows=rows).items()}
    before = d["residual"].clone()
    with pytest.raises(g4.G4Error) as e:
        g4.decoder_feedforward_noalloc(*[d[k] for k in MLP_ARGS])
    assert e.value.code == 6 and "limit" in str(e.value)
    torch.cuda.synchronize()
    assert torch.equal(d["residual"], before)
