"""The batched prefill's quantisation recipe in the oracle, without a GPU: its E4M3 and
E2M1 rounding against torch's float8 conversion and the library's weight quantiser,
per-row NVFP4 against quantize_nvfp4 applied row by row, the zero-row case, and the
size of the NVFP4-activation effect on one token of the reference MLP."""

import numpy as np
import pytest
import torch

from g4formats import quant
from oracle import ops, prng


def test_e4m3_round_matches_torch_float8():
    v = np.abs(np.random.default_rng(0).standard_normal(50000).astype(np.float32)) * np.float32(40)
    mids = (ops._E4M3_POS[1:] + ops._E4M3_POS[:-1]) / 2  # exact ties
    v = np.concatenate([v, ops._E4M3_POS, mids, [448.0, 449.0, 1e6, 0.0]]).astype(np.float32)
    want = torch.from_numpy(np.minimum(v, 448.0)).to(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(ops.e4m3_round(v), want)


def test_e2m1_round_matches_the_weight_quantiser():
    w = np.random.default_rng(1).standard_normal(50000).astype(np.float32) * 3
    ties = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0], dtype=np.float32)
    w = np.concatenate([w, ties, -ties]).astype(np.float32)
    codes = quant.e2m1_encode(torch.from_numpy(w)).numpy()
    want = prng.E2M1_MAGNITUDE[codes & 7] * np.where(codes >= 8, -1.0, 1.0)
    np.testing.assert_array_equal(ops.e2m1_round(w) + 0.0, want.astype(np.float32) + 0.0)


def test_row_quantiser_is_the_weight_recipe_per_row():
    x = prng.round_bf16(np.random.default_rng(2).standard_normal((4, 3840)).astype(np.float32))
    x[3] *= np.float32(1e-3)
    xq, ginv = ops.nvfp4_quantize_rows(x)
    for r in range(4):
        p, s, rec = quant.quantize_nvfp4(torch.from_numpy(x[r:r + 1]))
        np.testing.assert_array_equal(ops.nvfp4_dequant(p.numpy(), s.numpy())[0], xq[r])
        assert float(rec[0]) == float(ginv[r])


def test_row_quantiser_zero_row():
    x = np.zeros((2, 64), dtype=np.float32)
    x[1, 5] = 3.0
    xq, ginv = ops.nvfp4_quantize_rows(x)
    assert not np.any(xq[0]) and ginv[0] == 0.0
    assert xq[1, 5] * ginv[1] == pytest.approx(3.0, rel=1e-6)  # the row's max is exact


def test_more_pieces_shrink_the_error():
    x = prng.round_bf16(np.random.default_rng(3).standard_normal((16, 3840)).astype(np.float32))
    errs = []
    for p in (1, 2, 3):
        xq, ginv = ops.nvfp4_quantize_rows(x, p)
        errs.append(float(np.linalg.norm(xq * ginv[:, None] - x) / np.linalg.norm(x)))
    assert errs[0] < 0.15 and errs[1] < 0.02 and errs[2] < 0.003, errs


@pytest.mark.slow
def test_prefill_oracle_is_close_to_the_reference_mlp():
    """One token: the NVFP4-activation recipe against the reference's bf16 MLP.  Two
    pieces keep the output within the reference tolerance (max-abs 2e-2, rel-L2 1e-2)."""
    m = quant.mlp_config1(seed=4, device="cpu")
    H, L = ops.H, ops.L
    deq = {n: ops.nvfp4_dequant(m[f"{n}_weight_packed"].numpy().reshape(r, k // 2),
                                m[f"{n}_weight_scale"].numpy().reshape(r, k // 16))
           for n, r, k in (("gate", L, H), ("up", L, H), ("down", H, L))}
    f = lambda t: t.float().numpy().reshape(-1)  # noqa: E731
    gs = [np.float32(m[f"{n}_global_scale"][0]) for n in ("up", "gate", "down")]
    res = f(m["residual"])
    ref = ops.decoder_feedforward(
        res, f(m["pre_ff_rms_weight"]), f(m["post_ff_rms_weight"]), m["up_weight_packed"].numpy().reshape(L, H // 2),
        m["gate_weight_packed"].numpy().reshape(L, H // 2), m["down_weight_packed"].numpy().reshape(H, L // 2),
        m["up_weight_scale"].numpy().reshape(L, -1), m["gate_weight_scale"].numpy().reshape(L, -1),
        m["down_weight_scale"].numpy().reshape(H, -1), *gs, f(m["layer_scalar"])[0])
    rels = {}
    for p in (1, 2):
        q = ops.prefill_feedforward(res[None], f(m["pre_ff_rms_weight"]), f(m["post_ff_rms_weight"]), deq["up"],
                                    deq["gate"], deq["down"], *gs, f(m["layer_scalar"])[0], pieces=p)[0]
        a, b = ref - res, q - res
        rels[p] = float(np.linalg.norm(a - b) / np.linalg.norm(a))
        if p == 2:
            assert float(np.abs(q - ref).max()) <= 2e-2
            assert float(np.linalg.norm(q - ref) / np.linalg.norm(ref)) <= 1e-2
    print("NVFP4-activation effect on one token's MLP contribution (rel-L2) by pieces:", rels)
    assert 0.0 < rels[1] < 0.25 and rels[2] < 0.03
