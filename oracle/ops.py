"""CPU oracle for the text-decoder hot path: numpy restatements of the reference math.

TEST INFRASTRUCTURE ONLY (the checker): used by tests/, `__graft_entry__.smoke()` and the
CPU-baseline leg of bench.py.  The shipped CUDA path never imports this package.

Each function restates, in float32 numpy with explicit bf16 rounding at exactly the
points where the reference's torch code rounds, one kernel of the reference's own
expected-output generator (scripts/generate_references.py) and its building blocks
(transformers Gemma4 modules it instantiates).  Rounding points:
  - RMSNorm: f32 x * pow(mean(x^2)+eps, -0.5) [* w]  -> bf16          (Gemma4RMSNorm)
  - FP8 projection: bf16((x.float() @ codes.T) * scale)               (:312-321)
  - NVFP4 projection: bf16(bf16(x @ W.T) * global)                     (:588-602)
  - bf16 elementwise ops (RoPE products/sum, GELU, residual add, gate): one bf16
    rounding per torch op, computed in f32.
"""

from __future__ import annotations

import numpy as np

from . import prng

H, L, W = 3840, 15360, 262144
NS, GS, DS, QS, PS, TS = 8, 2, 256, 4096, 2048, 1024
GF, DF, QF, PF, TF = 16, 512, 8192, 512, 512
E = 32768
EPS = np.float32(1e-6)
EMBED_SCALE = 61.967734
LOGIT_SOFTCAP = np.float32(30.0)

f32 = np.float32
rb = prng.round_bf16


def as_f32(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> float32 values."""
    return prng.bf16_to_f32(bits)


def rms_norm(x: np.ndarray, weight: np.ndarray | None, eps: np.float32 = EPS) -> np.ndarray:
    """Gemma4RMSNorm over the last axis (transformers gemma4; scripts/gemma4.py:80-94).

    x, weight: float32 arrays holding bf16 values.  Returns bf16-rounded float32.
    torch.pow(ms, -0.5) on CPU is 1/sqrt(ms) with both steps correctly rounded.
    """
    x = np.asarray(x, dtype=f32)
    ms = (x * x).astype(f32).sum(axis=-1, keepdims=True, dtype=np.float64).astype(f32)
    ms = (ms / f32(x.shape[-1])).astype(f32) + eps
    r = (f32(1.0) / np.sqrt(ms.astype(f32))).astype(f32)
    y = (x * r).astype(f32)
    if weight is not None:
        y = (y * np.asarray(weight, dtype=f32)).astype(f32)
    return rb(y)


def scaled_projection(x: np.ndarray, codes_f8: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """bf16((x @ codes.T) * scale) -- generate_references.py:312-321 (f32 contraction)."""
    w = prng.e4m3_decode(codes_f8).astype(f32)
    acc = (w @ np.asarray(x, dtype=f32)).astype(f32)
    return rb(acc * np.asarray(scale, dtype=f32))


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """apply_rotary_pos_emb with bf16 tensors: bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)).

    cos/sin are the UNMODIFIED (upstream-convention) bf16 tables of one position
    (generate_references.py:405-408, transformers apply_rotary_pos_emb/rotate_half).
    """
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return rb(rb(x * cos) + rb(rot * sin))


def rope_tables(head_dim: int, theta: float, factor: float, pos: int):
    """f64 cos/sin of one position, narrowed to f32 (generate_references.py:243-257)."""
    angles = int(factor * head_dim // 2)
    inv = 1.0 / (np.float64(theta) ** (np.arange(0, 2 * angles, 2, dtype=np.float64) / head_dim))
    inv = np.concatenate([inv, np.zeros(head_dim // 2 - angles)])
    emb = np.concatenate([pos * inv, pos * inv])
    return np.cos(emb).astype(f32), np.sin(emb).astype(f32)


def negate_low_half(sin: np.ndarray) -> np.ndarray:
    """The kernel-side sin operand (generate_references.py:260-270)."""
    out = np.array(sin, dtype=f32, copy=True)
    out[: out.shape[-1] // 2] *= -1.0
    return out


# ---------------------------------------------------------------------------- per kernel
def embed_token(row: np.ndarray) -> np.ndarray:
    """bf16(row * bf16(EMBED_SCALE)) -- Gemma4TextScaledWordEmbedding (:347-368)."""
    return rb(np.asarray(row, dtype=f32) * rb(np.array([EMBED_SCALE], dtype=f32))[0])


def project_sliding(x, input_w, q_codes, k_codes, v_codes, q_scale, k_scale, v_scale,
                    q_norm_w, k_norm_w, cos, sin):
    """_project_sliding (generate_references.py:379-425) -> (q[NS*GS,DS], k[NS,DS], v[NS,DS]).

    Head counts follow the weight shapes, so a tensor-parallel shard restates too.
    """
    h = rms_norm(x, input_w)
    q = rms_norm(scaled_projection(h, q_codes, q_scale).reshape(-1, DS), q_norm_w)
    q = rope(q, cos, sin)
    k = rms_norm(scaled_projection(h, k_codes, k_scale).reshape(-1, DS), k_norm_w)
    k = rope(k, cos, sin)
    v = rms_norm(scaled_projection(h, v_codes, v_scale).reshape(-1, DS), None)
    return q, k, v


def project_full(x, input_w, q_codes, k_codes, q_scale, k_scale, q_norm_w, k_norm_w, cos, sin):
    """_project_full (generate_references.py:480-521): MQA, V = unweighted norm of raw K."""
    h = rms_norm(x, input_w)
    q = rms_norm(scaled_projection(h, q_codes, q_scale).reshape(-1, DF), q_norm_w)
    q = rope(q, cos, sin)
    k_raw = scaled_projection(h, k_codes, k_scale).reshape(DF)
    k = rope(rms_norm(k_raw, k_norm_w), cos, sin)
    v = rms_norm(k_raw, None)
    return q, k, v


def masked_softmax_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, mask: np.ndarray) -> np.ndarray:
    """softmax(q k^T masked, scale 1) v in f32 -> bf16 (generate_references.py:324-330,436-455).

    q [heads, D], k/v [T, D] (one kv head), mask [T] (>0 = attended).
    """
    s = (np.asarray(q, dtype=np.float64) @ np.asarray(k, dtype=np.float64).T).astype(f32)
    valid = np.asarray(mask) > 0
    s = np.where(valid[None, :], s, -np.inf).astype(f32)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp((s - m).astype(f32)).astype(f32)
    p = (e / e.sum(axis=-1, keepdims=True, dtype=np.float64).astype(f32)).astype(f32)
    return rb((p.astype(np.float64) @ np.asarray(v, dtype=np.float64)).astype(f32))


def sliding_attention(q, k_cache, v_cache, mask):
    """gen_sliding_attention: q [NS,GS,DS], caches [TS,NS,DS], mask [TS] -> [NS,GS,DS]."""
    nkv = q.shape[0]
    out = np.empty(q.shape, dtype=f32)
    for n in range(nkv):
        out[n] = masked_softmax_attention(q[n], k_cache[:, n, :], v_cache[:, n, :], mask)
    return out


def attention_output(x_flat, o_codes, o_scale, post_w, residual):
    """_attention_output_sliding (generate_references.py:458-469)."""
    projected = scaled_projection(x_flat, o_codes, o_scale)
    return rb(np.asarray(residual, dtype=f32) + rms_norm(projected, post_w))


def full_attention_output(x, running_sum, o_codes, o_scale, post_w, residual):
    """_attention_output_full (generate_references.py:559-577): x/sum then o-proj."""
    nx = rb(np.asarray(x, dtype=f32) / np.asarray(running_sum, dtype=f32)[:, None])
    return attention_output(nx.reshape(-1), o_codes, o_scale, post_w, residual)


def nvfp4_dequant(packed: np.ndarray, block_scale: np.ndarray) -> np.ndarray:
    """codes * local.repeat_interleave(16) in f32, exact in bf16 (:622-626)."""
    vals = prng.e2m1_unpack(packed)
    sc = prng.e4m3_decode(block_scale).astype(f32)
    return (vals * np.repeat(sc, 16, axis=-1)).astype(f32)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    """gelu(x, approximate='tanh') in f32 (torch's CPU formula)."""
    x = np.asarray(x, dtype=f32)
    inner = f32(0.7978845608028654) * (x + f32(0.044715) * (x * x * x))
    return (f32(0.5) * x * (f32(1.0) + np.tanh(inner.astype(f32)))).astype(f32)


def globally_scaled_linear(x: np.ndarray, w: np.ndarray, gscale: np.float32) -> np.ndarray:
    """GloballyScaled(nn.Linear) in bf16: bf16(bf16(x @ W.T) * s) (:588-602)."""
    acc = (w.astype(f32) @ np.asarray(x, dtype=f32)).astype(f32)
    return rb(rb(acc) * f32(gscale))


def decoder_feedforward(residual, pre_w, post_w, up_p, gate_p, down_p, up_s, gate_s, down_s,
                        up_gs, gate_gs, down_gs, layer_scalar):
    """gen_decoder_feedforward (generate_references.py:605-639), one token."""
    hidden = rms_norm(residual, pre_w)
    gate = globally_scaled_linear(hidden, nvfp4_dequant(gate_p, gate_s), gate_gs)
    up = globally_scaled_linear(hidden, nvfp4_dequant(up_p, up_s), up_gs)
    act = rb(rb(gelu_tanh(gate)) * up)
    down = globally_scaled_linear(act, nvfp4_dequant(down_p, down_s), down_gs)
    hidden = rms_norm(down, post_w)
    return rb(rb(np.asarray(residual, dtype=f32) + hidden) * f32(layer_scalar))


def final_norm_and_logits(x, rms_w, lm_head_bits: np.ndarray, rows_per_block: int = 4096):
    """gen_final_norm_and_logits (generate_references.py:642-669): f32 GEMV -> bf16 -> softcap."""
    normed = rms_norm(x, rms_w).astype(f32)
    n = lm_head_bits.shape[0]
    logits = np.empty(n, dtype=f32)
    for s in range(0, n, rows_per_block):
        blk = as_f32(lm_head_bits[s:s + rows_per_block])
        logits[s:s + rows_per_block] = rb(blk @ normed)
    return softcap(logits)


def softcap(logits: np.ndarray) -> np.ndarray:
    return rb(np.tanh((np.asarray(logits, dtype=f32) / LOGIT_SOFTCAP).astype(f32)) * LOGIT_SOFTCAP)


# ---------------------------------------------------------------------------- batched prefill
# The reference prefills one position per dispatch (src/host/generate.rs:194-211) with
# bf16 activations.  The library's batched prefill MLP (g4_decoder_feedforward_prefill)
# feeds the block-scaled FP4 tensor cores, so it quantises each token's activations to
# NVFP4 with the checkpoint weights' own recipe.  `prefill_feedforward` restates that
# recipe around the reference MLP (decoder_feedforward above) so the CUDA path is checked
# against exactly what it computes; the tests compare it with the unquantised reference as
# well, to bound the quantisation's effect.

def _nearest_code(v: np.ndarray, grid: np.ndarray) -> np.ndarray:
    """Index of the nearest value of the ascending non-negative `grid` for v >= 0, ties
    to the even index (round-to-nearest-even when consecutive codes alternate parity)."""
    hi = np.clip(np.searchsorted(grid, v, side="left"), 1, len(grid) - 1)
    lo = hi - 1
    dlo, dhi = v - grid[lo], grid[hi] - v
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    idx = np.where(pick_hi, hi, lo)
    return np.where(v >= grid[-1], len(grid) - 1, idx)


_E4M3_POS = prng.E4M3_VALUE[:127].astype(f32)  # codes 0x00..0x7E, ascending, 0..448


def e4m3_round(v: np.ndarray) -> np.ndarray:
    """Non-negative f32 -> nearest E4M3 value (ties to even, saturating at 448)."""
    v = np.asarray(v, dtype=f32)
    return _E4M3_POS[_nearest_code(np.minimum(v, f32(448.0)), _E4M3_POS)]


def e2m1_round(v: np.ndarray) -> np.ndarray:
    """f32 -> nearest E2M1 value (ties to even, saturating at +/-6)."""
    v = np.asarray(v, dtype=f32)
    mag = prng.E2M1_MAGNITUDE[_nearest_code(np.abs(v), prng.E2M1_MAGNITUDE)]
    return np.where(v < 0, -mag, mag).astype(f32)


def nvfp4_quantize_rows(x: np.ndarray, pieces: int = 1):
    """Per row of x [T, K] (bf16 values), `pieces` NVFP4 rows sharing one scale
    g = reciprocal(max|row|) * 2688: with y_0 = x * g,
      s_p = e4m3(max_b|y_p| / 6)   (p = 0: e4m3(max_b|x| / 6 * g), the weight recipe),
      c_p = e2m1(y_p / s_p),       y_{p+1} = y_p - c_p * s_p.
    Returns the pieces' values the MMA sees, sum_p c_p * s_p (in f32), and 1/g per row
    (0 for an all-zero row)."""
    x = np.asarray(x, dtype=f32)
    t, k = x.shape
    amax = np.abs(x).max(axis=1)
    zero = ~(amax > 0) | ~np.isfinite(amax)
    safe = np.where(zero, f32(1.0), amax).astype(f32)
    g = np.where(zero, f32(1.0), ((f32(1.0) / safe).astype(f32) * f32(2688.0)).astype(f32)).astype(f32)
    blocks = x.reshape(t, k // 16, 16)
    y = (blocks * g[:, None, None]).astype(f32)
    smax = ((np.abs(blocks).max(axis=2) / f32(6.0)).astype(f32) * g[:, None]).astype(f32)
    total = np.zeros_like(y)
    for p in range(pieces):
        if p > 0:
            smax = (np.abs(y).max(axis=2) / f32(6.0)).astype(f32)
        s = e4m3_round(smax)
        s = np.where(zero[:, None], f32(0.0), s).astype(f32)
        with np.errstate(divide="ignore", invalid="ignore"):
            scaled = (y / s[:, :, None]).astype(f32)
        piece = (np.where(s[:, :, None] > 0, e2m1_round(scaled), f32(0.0)) * s[:, :, None]).astype(f32)
        y = (y - piece).astype(f32)
        total = (total + piece).astype(f32)
    ginv = np.where(zero, f32(0.0), (f32(1.0) / g).astype(f32)).astype(f32)
    return total.reshape(t, k), ginv


def prefill_feedforward(residual, pre_w, post_w, up_w, gate_w, down_w, up_gs, gate_gs, down_gs, layer_scalar,
                        pieces: int = 2, world: int = 1):
    """decoder_feedforward for T tokens [T, H] with activations as `pieces` NVFP4 pieces
    (nvfp4_quantize_rows).  The weights are dequantised (nvfp4_dequant) f32 [rows, K];
    global scales are the reciprocals the kernels take.  Rounding points as
    decoder_feedforward, with x @ W.T replaced by (q(x) @ W.T) / g.  world > 1: the
    tensor-parallel split, h quantised per rank's column slice and the ranks' down sums
    (each divided by its own g) added in f32 before the bf16 roundings."""
    res = np.asarray(residual, dtype=f32)
    hidden = rms_norm(res, pre_w)
    xq, gx = nvfp4_quantize_rows(hidden, pieces)

    def proj(a, w, ginv, gs):
        acc = (a @ w.T).astype(f32)
        return rb(rb((acc * ginv[:, None]).astype(f32)) * f32(gs))

    gate = proj(xq, gate_w, gx, gate_gs)
    up = proj(xq, up_w, gx, up_gs)
    act = rb(rb(gelu_tanh(gate)) * up)
    lr = act.shape[1] // world
    ysum = np.zeros((act.shape[0], down_w.shape[0]), dtype=f32)
    for r in range(world):
        hq, gh = nvfp4_quantize_rows(act[:, r * lr:(r + 1) * lr], pieces)
        part = ((hq @ down_w[:, r * lr:(r + 1) * lr].T).astype(f32) * gh[:, None]).astype(f32)
        ysum = (ysum + part).astype(f32)
    down = rb(rb(ysum) * f32(down_gs))
    hidden = rms_norm(down, post_w)
    return rb(rb(res + hidden) * f32(layer_scalar))
