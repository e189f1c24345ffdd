"""GPU test harness: runs the reference's kernel cases through the C ABI.

Inputs come from the oracle's case builders (byte-identical to the reference's
synthesis) and are laid out exactly as the reference's Rust test shims lay them out
(src/bin/test_kernels.rs:522-893); each `run_<case>` returns the same labelled outputs
the reference test reads back.  The 2 GB lm_head is synthesized on the device with a
torch restatement of the same name-hashed stream (verified against the reference's
recorded checksum).
"""

from __future__ import annotations

import numpy as np
import torch

import g4b200 as g4
from oracle import cases, ops, prng

DEV = "cuda"


def t_bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(DEV)


def t_u8(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint8)).to(DEV)


def t_f32(a) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(DEV)


def t_i32(a) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int32)).to(DEV)


def to_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().reshape(-1)


def zeros_bf16(n: int) -> torch.Tensor:
    return torch.zeros(n, dtype=torch.bfloat16, device=DEV)


# --------------------------------------------------------------- device-side synthesis
_MASK = (1 << 64) - 1


def _i64(v: int) -> int:
    v &= _MASK
    return v - (1 << 64) if v >= (1 << 63) else v


def _lsr(z: torch.Tensor, k: int) -> torch.Tensor:
    return (z >> k) & ((1 << (64 - k)) - 1)


def t_words(name: str, first: int, count: int) -> torch.Tensor:
    """fixture_prng words on the device (int64 arithmetic wraps like uint64)."""
    z = torch.arange(first, first + count, dtype=torch.int64, device=DEV) ^ _i64(prng.name_seed(name))
    z = z + _i64(0x9E3779B97F4A7C15)
    z = (z ^ _lsr(z, 30)) * _i64(0xBF58476D1CE4E5B9)
    z = (z ^ _lsr(z, 27)) * _i64(0x94D049BB133111EB)
    return z ^ _lsr(z, 31)


def t_bf16_uniform(name: str, first: int, count: int, lo: float, hi: float) -> torch.Tensor:
    """bf16 bits (as int32) of lo + (hi-lo)*u, one f32 multiply then one add."""
    u = _lsr(t_words(name, first, count), 40).to(torch.float32) * (1.0 / 16777216.0)
    lo32, span = np.float32(lo), np.float32(np.float32(hi) - np.float32(lo))
    f = (u * float(span)) + float(lo32)
    bits = f.view(torch.int32)
    return ((bits + (0x7FFF + ((bits >> 16) & 1))) >> 16) & 0xFFFF


def t_checksum(bits16: torch.Tensor, word_offset: int) -> int:
    """Position-weighted u32 checksum of a bf16 bit stream (pairs packed little-endian)."""
    b = bits16.to(torch.int64).view(-1, 2)
    w = b[:, 0] | (b[:, 1] << 16)
    idx = torch.arange(w.numel(), dtype=torch.int64, device=w.device) + word_offset
    return int(((w * ((idx * 2 + 1) & 0xFFFFFFFF)) & 0xFFFFFFFF).sum().item()) & 0xFFFFFFFF


def device_lm_head(name: str = "final_norm_and_logits.lm_head_weight", rows: int = ops.W):
    """The [rows, H] lm_head synthesized on the GPU, plus its reference-style checksum."""
    out = torch.empty(rows * ops.H, dtype=torch.int16, device=DEV)
    step = max(1, (1 << 23) // ops.H)
    total = 0
    for s in range(0, rows, step):
        n = min(step, rows - s)
        bits = t_bf16_uniform(name, s * ops.H, n * ops.H, *cases.CENTRED)
        total = (total + t_checksum(bits, s * ops.H // 2)) & 0xFFFFFFFF
        out[s * ops.H:(s + n) * ops.H] = bits.to(torch.int32).to(torch.int16)
    return out.view(torch.bfloat16), total


# --------------------------------------------------------------- case runners
def run_embed_token(ctx, c):
    table = zeros_bf16(ops.W * ops.H)
    tok = c.inputs["token"]
    table[tok * ops.H:(tok + 1) * ops.H] = t_bf16(c.inputs["row"])
    out = zeros_bf16(ops.H)
    g4.embed_token(ctx, table, t_i32(c.inputs["offset"]), out)
    torch.cuda.synchronize()
    return {"expected": to_f32(out)}


def run_copy_hidden_state(ctx, c):
    out = zeros_bf16(ops.H)
    g4.copy_hidden_state(ctx, t_bf16(c.inputs["x"]), out)
    torch.cuda.synchronize()
    return {"expected": to_f32(out)}


def run_sliding_project_qkv(ctx, c):
    i = c.inputs
    x = i.get("x_exact", i["x_signs"])
    kc, vc, q = zeros_bf16(ops.TS * ops.NS * ops.DS), zeros_bf16(ops.TS * ops.NS * ops.DS), zeros_bf16(ops.QS)
    g4.sliding_project_qkv(ctx, t_bf16(x), t_u8(i["q_weight"]), t_u8(i["k_weight"]), t_u8(i["v_weight"]),
                           t_bf16(i["q_weight_scale"]), t_bf16(i["k_weight_scale"]), t_bf16(i["v_weight_scale"]),
                           t_bf16(i["input_rms_weight"]), t_bf16(i["q_rms_weight"]), t_bf16(i["k_rms_weight"]),
                           t_i32(i["kv_offset"]), t_i32(i["rope_offset"]), t_bf16(i["cos_table"]),
                           t_bf16(i["sin_table"]), kc, vc, q)
    torch.cuda.synchronize()
    w = ops.NS * ops.DS
    s = i["slot"]
    return {"expected.q": to_f32(q), "expected.k": to_f32(kc)[s * w:(s + 1) * w],
            "expected.v": to_f32(vc)[s * w:(s + 1) * w], "_caches": (kc, vc)}


def run_full_project_qkv(ctx, c):
    i = c.inputs
    x = i.get("x_exact", i["x_signs"])
    kc, vc, q = zeros_bf16(ops.TF * ops.DF), zeros_bf16(ops.TF * ops.DF), zeros_bf16(ops.QF)
    g4.full_project_qkv(ctx, t_bf16(x), t_u8(i["q_weight"]), t_u8(i["k_weight"]), t_bf16(i["q_weight_scale"]),
                        t_bf16(i["k_weight_scale"]), t_bf16(i["input_rms_weight"]), t_bf16(i["q_rms_weight"]),
                        t_bf16(i["k_rms_weight"]), t_i32(i["kv_offset"]), t_i32(i["rope_offset"]),
                        t_bf16(i["cos_table"]), t_bf16(i["sin_table"]), kc, vc, q)
    torch.cuda.synchronize()
    r = i["row"]
    return {"expected.q": to_f32(q), "expected.k": to_f32(kc)[r * ops.DF:(r + 1) * ops.DF],
            "expected.v": to_f32(vc)[r * ops.DF:(r + 1) * ops.DF], "_caches": (kc, vc)}


def run_sliding_attention(ctx, c):
    i = c.inputs
    out = zeros_bf16(ops.NS * ops.GS * ops.DS)
    g4.sliding_attention(ctx, t_bf16(i["q"]), t_bf16(i["k"]), t_bf16(i["v"]), t_f32(i["mask"]), out)
    torch.cuda.synchronize()
    return {"expected": to_f32(out)}


def run_full_attention(ctx, c):
    i = c.inputs
    rmax = torch.zeros(ops.GF, dtype=torch.float32, device=DEV)
    rsum = torch.zeros(ops.GF, dtype=torch.float32, device=DEV)
    out = zeros_bf16(ops.GF * ops.DF)
    q = t_bf16(i["q"])
    g4.full_attention_first_page(ctx, q, t_bf16(i["k0"]), t_bf16(i["v0"]), t_f32(i["mask0"]), rmax, rsum, out)
    g4.full_attention_page(ctx, q, t_bf16(i["k1"]), t_bf16(i["v1"]), t_f32(i["mask1"]), rmax, rsum, out)
    torch.cuda.synchronize()
    sums = rsum.cpu().numpy()
    vals = to_f32(out).reshape(ops.GF, ops.DF) / sums[:, None]
    return {"expected": vals.reshape(-1)}


def run_sliding_attention_output(ctx, c):
    i = c.inputs
    res = t_bf16(i["residual"])
    g4.sliding_attention_output(ctx, t_bf16(i["x"]), t_bf16(i["post_attn_rms_weight"]), t_u8(i["o_weight"]),
                                t_bf16(i["o_weight_scale"]), res)
    torch.cuda.synchronize()
    return {"expected": to_f32(res)}


def run_full_attention_output(ctx, c):
    i = c.inputs
    res = t_bf16(i["residual"])
    g4.full_attention_output(ctx, t_bf16(i["x"]), t_f32(i["running_sum"]), t_bf16(i["post_attn_rms_weight"]),
                             t_u8(i["o_weight"]), t_bf16(i["o_weight_scale"]), res)
    torch.cuda.synchronize()
    return {"expected": to_f32(res)}


def mlp_tensors(c):
    i = c.inputs
    return dict(
        residual=t_bf16(i["residual"]), pre_ff_rms_weight=t_bf16(i["pre_ff_rms_weight"]),
        up_weight_packed=t_u8(i["up_weight_packed"]), gate_weight_packed=t_u8(i["gate_weight_packed"]),
        down_weight_packed=t_u8(i["down_weight_packed"]), up_weight_scale=t_u8(i["up_weight_scale"]),
        gate_weight_scale=t_u8(i["gate_weight_scale"]), down_weight_scale=t_u8(i["down_weight_scale"]),
        up_global_scale=t_f32(i["up_global_scale"]), gate_global_scale=t_f32(i["gate_global_scale"]),
        down_global_scale=t_f32(i["down_global_scale"]), post_ff_rms_weight=t_bf16(i["post_ff_rms_weight"]),
        layer_scalar=t_bf16(i["layer_scalar"]))


def run_decoder_feedforward(ctx, c):
    t = mlp_tensors(c)
    g4.decoder_feedforward(ctx, **t)
    torch.cuda.synchronize()
    return {"expected": to_f32(t["residual"])}


def run_final_norm_and_logits(ctx, c):
    i = c.inputs
    lm, chk = device_lm_head()
    out = zeros_bf16(ops.W)
    g4.final_norm_and_logits(ctx, t_bf16(i["x"]), t_bf16(i["rms_weight"]), lm, out)
    torch.cuda.synchronize()
    return {"expected": to_f32(out), "_lm_checksum": chk}


RUNNERS = {
    "embed_token": run_embed_token,
    "copy_hidden_state": run_copy_hidden_state,
    "sliding_project_qkv_exact": run_sliding_project_qkv,
    "sliding_project_qkv_random": run_sliding_project_qkv,
    "sliding_attention": run_sliding_attention,
    "sliding_attention_output_exact": run_sliding_attention_output,
    "sliding_attention_output_random": run_sliding_attention_output,
    "full_project_qkv_exact": run_full_project_qkv,
    "full_project_qkv_random": run_full_project_qkv,
    "full_attention": run_full_attention,
    "full_attention_output_exact": run_full_attention_output,
    "full_attention_output_random": run_full_attention_output,
    "decoder_feedforward": run_decoder_feedforward,
    "final_norm_and_logits": run_final_norm_and_logits,
}


def build_case(name: str):
    """Inputs of a reference case; the heavy oracle outputs are not needed on the GPU
    side (the golden vectors are the expected values)."""
    if name == "decoder_feedforward":
        return cases.decoder_feedforward(with_expected=False)
    if name == "final_norm_and_logits":
        c = cases.Case("final_norm_and_logits")
        c.bf16("x", ops.H, cases.UNIT)
        c.bf16("rms_weight", ops.H, cases.UNIT)
        return c
    return cases.BUILDERS[name]()
