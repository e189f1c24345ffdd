"""Batched prefill MLP (g4_decoder_feedforward_prefill) on a B200.

The kernel writes each token's activations as 1-3 NVFP4 pieces for the block-scaled FP4
tensor cores; oracle/ops.py:prefill_feedforward restates exactly that recipe around the
reference MLP (generate_references.py:605-639 rounding points), so:
  - GPU vs that oracle, 1 and 2 pieces: the MLP's contribution (out - residual) within
    PREFILL_REL_L2 (summation order differs, and a rare activation code can round the
    other way);
  - GPU (2 pieces, the default) vs the reference's bf16-activation MLP
    (ops.decoder_feedforward, one token at a time): the output within the reference
    tolerance, max-abs 2e-2 and rel-L2 1e-2; 1 piece's larger effect is printed;
  - tokens are independent: a token's output is bit-identical whether it runs among
    4096 tokens (config 5's M) or alone, which checks the full size without a full-size
    oracle; repeats are bit-identical; zero rows and rows spanning many octaves work.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import g4b200 as g4
from g4formats import quant
from oracle import ops

pytestmark = pytest.mark.gpu

H, L = ops.H, ops.L
PREFILL_REL_L2 = 2e-2   # MLP contribution, GPU vs the quantised-activation oracle
REF_MAX_ABS, REF_REL_L2 = 2e-2, 1e-2  # output, GPU (2 pieces) vs the reference MLP
ORDER = ("pre_ff_rms_weight", "up_weight_packed", "gate_weight_packed", "down_weight_packed", "up_weight_scale",
         "gate_weight_scale", "down_weight_scale", "up_global_scale", "gate_global_scale", "down_global_scale",
         "post_ff_rms_weight", "layer_scalar")


@pytest.fixture(scope="module")
def weights():
    """Config-5 weights (NVFP4 from N(0, 0.02), norms N(0, 0.1), seed 4): the CPU copy,
    the dequantised f32 matrices for the oracle, and the device copy."""
    m = quant.mlp_config1(seed=4, device="cpu")
    deq = {}
    for name, rows, k in (("gate", L, H), ("up", L, H), ("down", H, L)):
        deq[name] = ops.nvfp4_dequant(m[f"{name}_weight_packed"].numpy().reshape(rows, k // 2),
                                      m[f"{name}_weight_scale"].numpy().reshape(rows, k // 16))
    dev = {k: m[k].cuda() for k in ORDER}
    return m, deq, dev


def _residual(n: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, H, generator=g).to(torch.bfloat16)


def _oracle(m, deq, res: torch.Tensor, pieces: int = 2) -> np.ndarray:
    f = lambda t: t.float().numpy()  # noqa: E731
    return ops.prefill_feedforward(f(res), f(m["pre_ff_rms_weight"]), f(m["post_ff_rms_weight"]), deq["up"],
                                   deq["gate"], deq["down"], np.float32(m["up_global_scale"][0]),
                                   np.float32(m["gate_global_scale"][0]), np.float32(m["down_global_scale"][0]),
                                   f(m["layer_scalar"])[0], pieces=pieces)


@pytest.fixture
def pctx(gpu_ctx, request):
    """The shared context with the requested piece count (restored to 2 afterwards)."""
    gpu_ctx.set_prefill_pieces(getattr(request, "param", 2))
    yield gpu_ctx
    gpu_ctx.set_prefill_pieces(2)


def _run(ctx, dev, res: torch.Tensor) -> torch.Tensor:
    d = res.cuda().contiguous().clone()
    g4.decoder_feedforward_prefill(ctx, d, *[dev[k] for k in ORDER])
    torch.cuda.synchronize()
    assert ctx.poll() == 0
    return d


def _contrib_rel_l2(res: torch.Tensor, want: np.ndarray, got: np.ndarray) -> float:
    r = res.float().numpy()
    a, b = want.reshape(r.shape) - r, got.reshape(r.shape) - r
    return float(np.linalg.norm(a - b) / np.linalg.norm(a))


@pytest.mark.parametrize("pctx", [1, 2, 3], indirect=True)
@pytest.mark.parametrize("n", [1, 130, 257])
def test_prefill_matches_quantised_oracle(pctx, weights, n):
    """Ragged token counts: one token, one full 128-token tile plus 2, two tiles plus 1."""
    m, deq, dev = weights
    pieces = pctx.prefill_pieces
    res = _residual(n, 100 + n)
    want = _oracle(m, deq, res, pieces)
    got = _run(pctx, dev, res).float().cpu().numpy()
    rel = _contrib_rel_l2(res, want, got)
    per_tok = [_contrib_rel_l2(res[i:i + 1], want[i:i + 1], got[i:i + 1]) for i in range(n)]
    print(f"pieces={pieces} n={n}: contribution rel-L2 {rel:.3e}, worst token {max(per_tok):.3e}")
    assert np.isfinite(got).all()
    assert rel <= PREFILL_REL_L2 and max(per_tok) <= 2 * PREFILL_REL_L2


def test_prefill_within_reference_tolerance(gpu_ctx, weights):
    """Two pieces (the default) against the reference's bf16-activation MLP, one token at a
    time: the output within max-abs 2e-2 and rel-L2 1e-2."""
    m, deq, dev = weights
    res = _residual(4, 77)
    gpu_ctx.set_prefill_pieces(2)
    got = _run(gpu_ctx, dev, res).float().cpu().numpy()
    gpu_ctx.set_prefill_pieces(1)
    got1 = _run(gpu_ctx, dev, res).float().cpu().numpy()
    gpu_ctx.set_prefill_pieces(2)
    a = {k: v for k, v in m.items()}
    f = lambda t: t.float().numpy().reshape(-1)  # noqa: E731
    rels, rels1 = [], []
    for i in range(4):
        want = ops.decoder_feedforward(
            res[i].float().numpy(), f(a["pre_ff_rms_weight"]), f(a["post_ff_rms_weight"]),
            a["up_weight_packed"].numpy().reshape(L, H // 2), a["gate_weight_packed"].numpy().reshape(L, H // 2),
            a["down_weight_packed"].numpy().reshape(H, L // 2), a["up_weight_scale"].numpy().reshape(L, -1),
            a["gate_weight_scale"].numpy().reshape(L, -1), a["down_weight_scale"].numpy().reshape(H, -1),
            np.float32(a["up_global_scale"][0]), np.float32(a["gate_global_scale"][0]),
            np.float32(a["down_global_scale"][0]), f(a["layer_scalar"])[0])
        rels.append(_contrib_rel_l2(res[i:i + 1], want[None], got[i:i + 1]))
        rels1.append(_contrib_rel_l2(res[i:i + 1], want[None], got1[i:i + 1]))
        d = np.abs(got[i] - want)
        assert float(d.max()) <= REF_MAX_ABS and float(np.linalg.norm(d) / np.linalg.norm(want)) <= REF_REL_L2, i
    print("MLP contribution rel-L2 vs the reference, 2 pieces:", [round(r, 4) for r in rels],
          "1 piece:", [round(r, 4) for r in rels1])


def test_prefill_full_size_tokens_are_independent(gpu_ctx, weights):
    """Config 5's M = 4096: sampled tokens equal the same tokens run alone, bit for bit,
    and match the oracle."""
    m, deq, dev = weights
    res = _residual(4096, 4)
    full = _run(gpu_ctx, dev, res)
    pick = [0, 1, 127, 128, 1000, 2047, 4000, 4095]
    alone = _run(gpu_ctx, dev, res[pick])
    assert torch.equal(full[pick], alone)
    want = _oracle(m, deq, res[pick])
    assert _contrib_rel_l2(res[pick], want, alone.float().cpu().numpy()) <= PREFILL_REL_L2
    again = _run(gpu_ctx, dev, res)
    assert torch.equal(full, again)  # deterministic


def test_prefill_zero_and_wide_range_rows(gpu_ctx, weights):
    m, deq, dev = weights
    g = torch.Generator().manual_seed(9)
    res = torch.randn(6, H, generator=g)
    res[0] = 0.0                                                     # all-zero row
    res[1] *= torch.pow(2.0, torch.randint(-20, 10, (H,), generator=g).float())  # many octaves
    res[2, ::7] = 0.0                                                # sparse zeros
    res[3] *= 1e4
    res[4] *= 1e-4
    res = res.to(torch.bfloat16)
    want = _oracle(m, deq, res)
    got = _run(gpu_ctx, dev, res).float().cpu().numpy()
    assert np.isfinite(got).all()
    assert np.array_equal(got[0], want[0])  # a zero row stays zero (no NaN from 0 * 1/0)
    for i in range(1, 6):
        rel = _contrib_rel_l2(res[i:i + 1], want[i:i + 1], got[i:i + 1])
        print(f"row {i}: contribution rel-L2 {rel:.3e}")
        assert rel <= 2 * PREFILL_REL_L2, (i, rel)


def test_prefill_argument_errors(gpu_ctx, weights):
    m, deq, dev = weights
    with pytest.raises(ValueError):
        g4.decoder_feedforward_prefill(gpu_ctx, torch.zeros(0, H, dtype=torch.bfloat16, device="cuda"),
                                       *[dev[k] for k in ORDER])
    import ctypes

    r = torch.zeros(2, H, dtype=torch.bfloat16, device="cuda")
    args = [r] + [dev[k] for k in ORDER]
    with pytest.raises(g4.G4Error):
        gpu_ctx.call("g4_decoder_feedforward_prefill", ctypes.c_int32(0), *args)
    with pytest.raises(g4.G4Error):
        gpu_ctx.call("g4_decoder_feedforward_prefill", ctypes.c_int32(g4.PREFILL_MAX_TOKENS + 1), *args)
    assert gpu_ctx.poll() == 0
