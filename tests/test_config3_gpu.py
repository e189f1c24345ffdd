"""BASELINE config 3 on a B200: one full-attention decode layer with NVFP4 projections
(full_project_qkv_nvfp4 -> attention over an 8192-position cache -> full_attention_output
_nvfp4 + residual), each stage against the oracle; and the synthetic geometry of 16 q
heads over 8 KV heads of 256 at 8192 positions (g4_attention_gqa).  Seed 2, x ~ N(0,1),
weights N(0, 0.02) quantized to NVFP4, KV cache ~ N(0,1)."""

import numpy as np
import pytest
import torch

import g4b200 as g4
from g4formats import quant
from oracle import cases, ops, prng

pytestmark = pytest.mark.gpu

POS = 8191  # the last row of page 15: the attention reads 16 full pages


def _bf16(gen, shape, std):
    return (torch.randn(shape, generator=gen) * std).to(torch.bfloat16)


def _np(t):
    return t.float().cpu().numpy()


def _check(label, want, got, atol):
    r = cases.compare(np.asarray(want, np.float32).reshape(-1), np.asarray(got, np.float32).reshape(-1), atol)
    print(label, r)
    assert r["ok"] and r["rel_l2"] <= 1e-2, (label, r)


def test_full_attention_layer_nvfp4_config3(gpu_ctx):
    gen = torch.Generator().manual_seed(2)
    x = _bf16(gen, (ops.H,), 1.0)
    w_in = (1.0 + torch.randn(ops.H, generator=gen) * 0.1).to(torch.bfloat16)
    qn = (1.0 + torch.randn(ops.DF, generator=gen) * 0.1).to(torch.bfloat16)
    kn = (1.0 + torch.randn(ops.DF, generator=gen) * 0.1).to(torch.bfloat16)
    post = (1.0 + torch.randn(ops.H, generator=gen) * 0.1).to(torch.bfloat16)
    mq = quant.quantize_nvfp4(torch.randn(ops.QF, ops.H, generator=gen) * 0.02)
    mk = quant.quantize_nvfp4(torch.randn(ops.PF, ops.H, generator=gen) * 0.02)
    mo = quant.quantize_nvfp4(torch.randn(ops.H, ops.QF, generator=gen) * 0.02)
    n_pages = POS // ops.TF + 1
    kp = [_bf16(gen, (ops.TF * ops.DF,), 1.0).cuda() for _ in range(n_pages)]
    vp = [_bf16(gen, (ops.TF * ops.DF,), 1.0).cuda() for _ in range(n_pages)]
    row = POS % ops.TF
    cos_raw, sin_raw = ops.rope_tables(ops.DF, 1_000_000.0, 0.25, POS)
    cos_t = np.zeros(ops.E * ops.DF, np.uint16)
    sin_t = np.zeros(ops.E * ops.DF, np.uint16)
    cos_t[POS * ops.DF:(POS + 1) * ops.DF] = prng.bf16_bits(cos_raw)
    sin_t[POS * ops.DF:(POS + 1) * ops.DF] = prng.bf16_bits(ops.negate_low_half(sin_raw))
    import harness

    d = lambda t: t.cuda()  # noqa: E731
    q_out = harness.zeros_bf16(ops.QF)
    g4.full_project_qkv_nvfp4(
        gpu_ctx, d(x), d(mq[0].reshape(-1)), d(mk[0].reshape(-1)), d(mq[1].reshape(-1)), d(mk[1].reshape(-1)),
        d(mq[2]), d(mk[2]), d(w_in), d(qn), d(kn), harness.t_i32([row * ops.DF * 2]),
        harness.t_i32([POS * ops.DF * 2]), harness.t_bf16(cos_t), harness.t_bf16(sin_t), kp[-1], vp[-1], q_out)
    torch.cuda.synchronize()
    # stage 1 oracle: GloballyScaled NVFP4 projections, per-head norms, partial RoPE
    h = ops.rms_norm(_np(x), _np(w_in))
    gsl = lambda m, v: ops.globally_scaled_linear(v, ops.nvfp4_dequant(m[0].numpy(), m[1].numpy()),  # noqa: E731
                                                  np.float32(m[2][0]))
    cos, sin = ops.as_f32(prng.bf16_bits(cos_raw)), prng.round_bf16(sin_raw)
    q = ops.rope(ops.rms_norm(gsl(mq, h).reshape(-1, ops.DF), _np(qn)), cos, sin)
    k_raw = gsl(mk, h)
    k = ops.rope(ops.rms_norm(k_raw, _np(kn)), cos, sin)
    v = ops.rms_norm(k_raw, None)
    _check("q", q, _np(q_out), 0.0625)
    _check("k", k, _np(kp[-1])[row * ops.DF:(row + 1) * ops.DF], 0.0625)
    _check("v", v, _np(vp[-1])[row * ops.DF:(row + 1) * ops.DF], 0.0625)
    # stage 2: every page in one launch, against the oracle's f32 softmax on the GPU's q/cache
    kpt = torch.tensor([t.data_ptr() for t in kp], dtype=torch.int64, device="cuda")
    vpt = torch.tensor([t.data_ptr() for t in vp], dtype=torch.int64, device="cuda")
    att = harness.zeros_bf16(ops.QF)
    rsum = torch.zeros(ops.GF, dtype=torch.float32, device="cuda")
    g4.full_attention_paged(gpu_ctx, q_out, kpt, vpt, n_pages, row, rsum, att)
    torch.cuda.synchronize()
    K = np.concatenate([_np(t) for t in kp]).reshape(-1, ops.DF)[:POS + 1]
    V = np.concatenate([_np(t) for t in vp]).reshape(-1, ops.DF)[:POS + 1]
    want_att = ops.masked_softmax_attention(_np(q_out).reshape(ops.GF, ops.DF), K, V, np.ones(POS + 1))
    _check("attention", want_att, _np(att), 2e-3)
    assert torch.equal(rsum.cpu(), torch.ones(ops.GF))
    # stage 3: NVFP4 o-proj, post-attention RMSNorm, residual add (in place)
    res = d(x).clone()
    g4.full_attention_output_nvfp4(gpu_ctx, att, rsum, d(post), d(mo[0].reshape(-1)), d(mo[1].reshape(-1)),
                                   d(mo[2]), res)
    torch.cuda.synchronize()
    proj = gsl(mo, _np(att))
    want = prng.round_bf16(_np(x) + ops.rms_norm(proj, _np(post)))
    _check("attention output", want, _np(res), 0.0625)
    assert gpu_ctx.poll() == 0


@pytest.mark.parametrize("valid", [8192, 5000])
def test_gqa_attention_8kv_heads_at_8192(gpu_ctx, valid):
    """16 q heads over 8 KV heads of 256 against an 8192-position cache ~ N(0,1)."""
    gen = torch.Generator().manual_seed(2)
    rows = 8192
    q = _bf16(gen, (ops.NS * ops.GS * ops.DS,), 1.0 / 16)
    k = _bf16(gen, (rows * ops.NS * ops.DS,), 1.0)
    v = _bf16(gen, (rows * ops.NS * ops.DS,), 1.0)
    mask = torch.zeros(rows, dtype=torch.float32)
    mask[:valid] = 1.0
    out = torch.zeros(ops.NS * ops.GS * ops.DS, dtype=torch.bfloat16, device="cuda")
    g4.attention_gqa(gpu_ctx, q.cuda(), k.cuda(), v.cuda(), mask.cuda(), out)
    torch.cuda.synchronize()
    want = ops.sliding_attention(_np(q).reshape(ops.NS, ops.GS, ops.DS), _np(k).reshape(rows, ops.NS, ops.DS),
                                 _np(v).reshape(rows, ops.NS, ops.DS), mask.numpy())
    _check(f"gqa {valid}", want, _np(out), 2e-3)
    assert gpu_ctx.poll() == 0
