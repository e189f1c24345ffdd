"""The reference's kernel test cases, synthesized input-for-input.

TEST INFRASTRUCTURE ONLY.  For each case name of the reference's test registry
(scripts/generate_references.py:762-782, src/bin/test_kernels.rs:399-495) this module
builds the kernel's inputs with the exact tensor names, value ranges and layouts the
reference uses -- the generator's `Synth` (:155-240) for the values, and the Rust test
shims (test_kernels.rs:522-893) for how they are laid out in device memory (whole
[E,D] RoPE tables with one row filled, zeroed caches, byte offsets) -- plus the
checksums the golden file records, and the oracle's expected outputs.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import ops, prng

# Value ranges and positions of the reference cases (generate_references.py:85-100).
RAW_GLOBAL_SCALES = {"up": 9600.0, "gate": 9600.0, "down": 12928.0}
WEIGHT_EXP = (7, 14)
LOCAL_SCALE_EXP = (8, 10)
ROW_SCALE = (0.0, 1e-3)
UNIT = (0.0, 1.0)
CENTRED = (-0.5, 0.5)
RMS_WEIGHT = (0.75, 1.25)
POS = 137
SLIDING_VALID = 300
FULL_ROW = 137
LAYER_SCALAR = 0.375
EMBED_TOKEN_ID = 90210


@dataclass
class Case:
    """Inputs (raw storage arrays), checksums and oracle outputs of one test case."""

    name: str
    inputs: dict = field(default_factory=dict)
    checks: dict = field(default_factory=dict)
    expected: dict = field(default_factory=dict)

    def seed(self, n: str) -> str:
        return f"{self.name}.{n}"

    def keep(self, n: str, storage: np.ndarray) -> np.ndarray:
        self.checks[n] = prng.checksum(storage)
        self.inputs[n] = storage
        return storage

    def bf16(self, n, count, span):
        return self.keep(n, prng.bf16_uniform(self.seed(n), count, *span))

    def signs(self, n, count, scale=1.0):
        return self.keep(n, prng.bf16_signs(self.seed(n), count, scale))

    def f8(self, n, count, band, signed=True):
        return self.keep(n, prng.f8_banded(self.seed(n), count, band[0], band[1], signed))

    def f4(self, n, count):
        return self.keep(n, prng.f4_nibbles(self.seed(n), count))

    def f32(self, n, count, span):
        return self.keep(n, prng.f32_uniform(self.seed(n), count, *span))

    def const_f32(self, n, values):
        return self.keep(n, np.ascontiguousarray(values, dtype=np.float32))

    def const_bf16(self, n, values):
        return self.keep(n, prng.bf16_bits(np.ascontiguousarray(values, dtype=np.float32)))

    def const_i32(self, n, value):
        return self.keep(n, np.array([value], dtype=np.int32))


def _rope_table_rows(c: Case, head_dim: int, theta: float, factor: float):
    """cos / kernel-sin rows at POS, and the whole [E, D] tables the shims upload."""
    cos_raw, sin_raw = ops.rope_tables(head_dim, theta, factor, POS)
    cos_row = c.const_bf16("cos", cos_raw)
    sin_row = c.const_bf16("sin", ops.negate_low_half(sin_raw))
    tables = {}
    for n, row in (("cos", cos_row), ("sin", sin_row)):
        t = np.zeros(ops.E * head_dim, dtype=np.uint16)
        t[POS * head_dim:(POS + 1) * head_dim] = row
        tables[n] = t
    # the oracle applies upstream's (unmodified) sin: generate_references.py:405-408
    return tables, ops.as_f32(cos_row), prng.round_bf16(sin_raw)


def _exact_or_signs(c: Case, exact: bool):
    w = c.bf16("input_rms_weight", ops.H, RMS_WEIGHT)
    signs = c.signs("x_signs", ops.H)
    if exact:  # x = bf16(signs / input_rms_weight), test_kernels.rs:306-322
        x = prng.bf16_bits(ops.as_f32(signs) / ops.as_f32(w))
        return c.keep("x_exact", x), w
    return signs, w


def sliding_project_qkv(name: str, exact: bool) -> Case:
    c = Case(name)
    x, w_in = _exact_or_signs(c, exact)
    qc = c.f8("q_weight", ops.QS * ops.H, WEIGHT_EXP)
    kc = c.f8("k_weight", ops.PS * ops.H, WEIGHT_EXP)
    vc = c.f8("v_weight", ops.PS * ops.H, WEIGHT_EXP)
    qs = c.bf16("q_weight_scale", ops.QS, ROW_SCALE)
    ks = c.bf16("k_weight_scale", ops.PS, ROW_SCALE)
    vs = c.bf16("v_weight_scale", ops.PS, ROW_SCALE)
    qn = c.bf16("q_rms_weight", ops.DS, UNIT)
    kn = c.bf16("k_rms_weight", ops.DS, UNIT)
    tables, cos, sin = _rope_table_rows(c, ops.DS, 10_000.0, 1.0)
    slot = POS % ops.TS
    c.const_i32("kv_offset", slot * ops.NS * ops.DS * 2)
    c.const_i32("rope_offset", POS * ops.DS * 2)
    c.inputs["cos_table"], c.inputs["sin_table"] = tables["cos"], tables["sin"]
    c.inputs["slot"] = slot
    q, k, v = ops.project_sliding(
        ops.as_f32(x), ops.as_f32(w_in), qc.reshape(ops.QS, ops.H), kc.reshape(ops.PS, ops.H),
        vc.reshape(ops.PS, ops.H), ops.as_f32(qs), ops.as_f32(ks), ops.as_f32(vs),
        ops.as_f32(qn), ops.as_f32(kn), cos, sin)
    c.expected = {"expected.q": q.reshape(-1), "expected.k": k.reshape(-1), "expected.v": v.reshape(-1)}
    return c


def full_project_qkv(name: str, exact: bool) -> Case:
    c = Case(name)
    x, w_in = _exact_or_signs(c, exact)
    qc = c.f8("q_weight", ops.QF * ops.H, WEIGHT_EXP)
    kc = c.f8("k_weight", ops.PF * ops.H, WEIGHT_EXP)
    qs = c.bf16("q_weight_scale", ops.QF, ROW_SCALE)
    ks = c.bf16("k_weight_scale", ops.PF, ROW_SCALE)
    qn = c.bf16("q_rms_weight", ops.DF, UNIT)
    kn = c.bf16("k_rms_weight", ops.DF, UNIT)
    tables, cos, sin = _rope_table_rows(c, ops.DF, 1_000_000.0, 0.25)
    c.const_i32("kv_offset", POS * ops.DF * 2)
    c.const_i32("rope_offset", POS * ops.DF * 2)
    c.inputs["cos_table"], c.inputs["sin_table"] = tables["cos"], tables["sin"]
    c.inputs["row"] = POS
    q, k, v = ops.project_full(
        ops.as_f32(x), ops.as_f32(w_in), qc.reshape(ops.QF, ops.H), kc.reshape(ops.PF, ops.H),
        ops.as_f32(qs), ops.as_f32(ks), ops.as_f32(qn), ops.as_f32(kn), cos, sin)
    c.expected = {"expected.q": q.reshape(-1), "expected.k": k.reshape(-1), "expected.v": v.reshape(-1)}
    return c


def sliding_attention() -> Case:
    c = Case("sliding_attention")
    q = c.signs("q", ops.NS * ops.GS * ops.DS, 1 / 16)
    k = c.signs("k", ops.TS * ops.NS * ops.DS)
    v = c.bf16("v", ops.TS * ops.NS * ops.DS, CENTRED)
    mask = np.zeros(ops.TS, dtype=np.float32)
    mask[:SLIDING_VALID] = 1.0
    c.const_f32("mask", mask)
    out = ops.sliding_attention(
        ops.as_f32(q).reshape(ops.NS, ops.GS, ops.DS), ops.as_f32(k).reshape(ops.TS, ops.NS, ops.DS),
        ops.as_f32(v).reshape(ops.TS, ops.NS, ops.DS), mask)
    c.expected = {"expected": out.reshape(-1)}
    return c


def full_attention() -> Case:
    c = Case("full_attention")
    q = c.signs("q", ops.GF * ops.DF, 1 / 16)
    k0 = c.signs("k0", ops.TF * ops.DF)
    k1 = c.signs("k1", ops.TF * ops.DF)
    v0 = c.bf16("v0", ops.TF * ops.DF, CENTRED)
    v1 = c.bf16("v1", ops.TF * ops.DF, CENTRED)
    m0 = c.const_f32("mask0", np.ones(ops.TF, dtype=np.float32))
    m1 = np.zeros(ops.TF, dtype=np.float32)
    m1[:FULL_ROW + 1] = 1.0
    m1 = c.const_f32("mask1", m1)
    k = np.concatenate([ops.as_f32(k0), ops.as_f32(k1)]).reshape(-1, ops.DF)
    v = np.concatenate([ops.as_f32(v0), ops.as_f32(v1)]).reshape(-1, ops.DF)
    out = ops.masked_softmax_attention(ops.as_f32(q).reshape(ops.GF, ops.DF), k, v, np.concatenate([m0, m1]))
    c.expected = {"expected": out.reshape(-1)}
    return c


def sliding_attention_output(name: str, exact: bool) -> Case:
    c = Case(name)
    n = ops.NS * ops.GS * ops.DS
    x = c.signs("x", n) if exact else c.bf16("x", n, CENTRED)
    post = c.bf16("post_attn_rms_weight", ops.H, UNIT)
    oc = c.f8("o_weight", ops.H * ops.QS, WEIGHT_EXP)
    osc = c.bf16("o_weight_scale", ops.H, ROW_SCALE)
    res = c.bf16("residual", ops.H, UNIT)
    out = ops.attention_output(ops.as_f32(x), oc.reshape(ops.H, ops.QS), ops.as_f32(osc), ops.as_f32(post),
                               ops.as_f32(res))
    c.expected = {"expected": out}
    return c


def full_attention_output(name: str, exact: bool) -> Case:
    c = Case(name)
    n = ops.GF * ops.DF
    x = c.signs("x", n) if exact else c.bf16("x", n, CENTRED)
    if exact:
        rs = c.const_f32("running_sum", np.full(ops.GF, 4.0, dtype=np.float32))
    else:
        rs = c.f32("running_sum", ops.GF, (2.0, 4.0))
    post = c.bf16("post_attn_rms_weight", ops.H, UNIT)
    oc = c.f8("o_weight", ops.H * ops.QF, WEIGHT_EXP)
    osc = c.bf16("o_weight_scale", ops.H, ROW_SCALE)
    res = c.bf16("residual", ops.H, UNIT)
    out = ops.full_attention_output(ops.as_f32(x).reshape(ops.GF, ops.DF), rs, oc.reshape(ops.H, ops.QF),
                                    ops.as_f32(osc), ops.as_f32(post), ops.as_f32(res))
    c.expected = {"expected": out}
    return c


def decoder_feedforward(with_expected: bool = True) -> Case:
    c = Case("decoder_feedforward")
    res = c.bf16("residual", ops.H, UNIT)
    pre = c.bf16("pre_ff_rms_weight", ops.H, UNIT)
    post = c.bf16("post_ff_rms_weight", ops.H, UNIT)
    ls = c.const_bf16("layer_scalar", np.full(8, LAYER_SCALAR, dtype=np.float32))
    w = {}
    for n, rows, cols in (("up", ops.L, ops.H), ("gate", ops.L, ops.H), ("down", ops.H, ops.L)):
        packed = c.f4(f"{n}_weight_packed", rows * cols).reshape(rows, cols // 2)
        scale = c.f8(f"{n}_weight_scale", rows * cols // 16, LOCAL_SCALE_EXP, signed=False).reshape(rows, cols // 16)
        gs = c.const_f32(f"{n}_global_scale", np.array([1.0 / RAW_GLOBAL_SCALES[n]], dtype=np.float32))
        w[n] = (packed, scale, gs)
    if with_expected:
        out = ops.decoder_feedforward(
            ops.as_f32(res), ops.as_f32(pre), ops.as_f32(post), w["up"][0], w["gate"][0], w["down"][0],
            w["up"][1], w["gate"][1], w["down"][1], w["up"][2][0], w["gate"][2][0], w["down"][2][0],
            ops.as_f32(ls)[0])
        c.expected = {"expected": out}
    return c


def embed_token() -> Case:
    c = Case("embed_token")
    row = c.bf16("row", ops.H, CENTRED)
    c.const_i32("offset", EMBED_TOKEN_ID * ops.H * 2)
    c.inputs["token"] = EMBED_TOKEN_ID
    c.expected = {"expected": ops.embed_token(ops.as_f32(row))}
    return c


def copy_hidden_state() -> Case:
    c = Case("copy_hidden_state")
    x = c.bf16("x", ops.H, CENTRED)
    c.expected = {"expected": ops.as_f32(x)}
    return c


def lm_head_weight(name: str = "final_norm_and_logits.lm_head_weight", rows: int = ops.W) -> np.ndarray:
    """The [W, H] bf16 lm_head of final_norm_and_logits, synthesized in row blocks."""
    out = np.empty(rows * ops.H, dtype=np.uint16)
    step = max(1, (1 << 23) // ops.H)
    for s in range(0, rows, step):
        n = min(step, rows - s)
        out[s * ops.H:(s + n) * ops.H] = prng.bf16_uniform(name, n * ops.H, *CENTRED, offset=s * ops.H)
    return out.reshape(rows, ops.H)


def lm_head_checksum(weight_bits: np.ndarray) -> int:
    """Block-summed checksum exactly as generate_references.py:656-666 accumulates it."""
    flat = weight_bits.reshape(-1)
    step = max(1, (1 << 23) // ops.H) * ops.H
    total = 0
    for s in range(0, flat.size, step):
        total = (total + prng.checksum(flat[s:s + step], word_offset=s // 2)) & 0xFFFFFFFF
    return total


def final_norm_and_logits(with_expected: bool = True) -> Case:
    c = Case("final_norm_and_logits")
    x = c.bf16("x", ops.H, UNIT)
    w = c.bf16("rms_weight", ops.H, UNIT)
    lm = lm_head_weight()
    c.inputs["lm_head_weight"] = lm
    c.checks["lm_head_weight"] = lm_head_checksum(lm)
    if with_expected:
        c.expected = {"expected": ops.final_norm_and_logits(ops.as_f32(x), ops.as_f32(w), lm)}
    return c


BUILDERS = {
    "embed_token": embed_token,
    "copy_hidden_state": copy_hidden_state,
    "sliding_project_qkv_exact": lambda: sliding_project_qkv("sliding_project_qkv_exact", True),
    "sliding_project_qkv_random": lambda: sliding_project_qkv("sliding_project_qkv_random", False),
    "sliding_attention": sliding_attention,
    "sliding_attention_output_exact": lambda: sliding_attention_output("sliding_attention_output_exact", True),
    "sliding_attention_output_random": lambda: sliding_attention_output("sliding_attention_output_random", False),
    "full_project_qkv_exact": lambda: full_project_qkv("full_project_qkv_exact", True),
    "full_project_qkv_random": lambda: full_project_qkv("full_project_qkv_random", False),
    "full_attention": full_attention,
    "full_attention_output_exact": lambda: full_attention_output("full_attention_output_exact", True),
    "full_attention_output_random": lambda: full_attention_output("full_attention_output_random", False),
    "decoder_feedforward": decoder_feedforward,
    "final_norm_and_logits": final_norm_and_logits,
}

# Tolerances of the reference's test table (src/bin/test_kernels.rs:397-495): pass iff
# every element has |got - want| <= atol + rtol*|want|.
RTOL = 2e-2
ATOL = {
    "copy_hidden_state": 0.0,
    "embed_token": 0.25,
    "sliding_project_qkv_exact": 0.0625,
    "sliding_project_qkv_random": 0.0625,
    "sliding_attention": 2e-3,
    "sliding_attention_output_exact": 0.1,
    "sliding_attention_output_random": 0.1,
    "full_project_qkv_exact": 0.0625,
    "full_project_qkv_random": 0.0625,
    "full_attention": 2e-3,
    "full_attention_output_exact": 0.0625,
    "full_attention_output_random": 0.0625,
    "decoder_feedforward": 0.02,
    "final_norm_and_logits": 0.125,
}


def compare(want: np.ndarray, got: np.ndarray, atol: float, rtol: float = RTOL) -> dict:
    """The reference's `compare` (test_kernels.rs:971-1016) plus the north-star metrics."""
    want = np.asarray(want, dtype=np.float32).reshape(-1)
    got = np.asarray(got, dtype=np.float32).reshape(-1)
    assert want.shape == got.shape, (want.shape, got.shape)
    diff = np.abs(want.astype(np.float64) - got.astype(np.float64))
    finite = bool(np.isfinite(got).all())
    within = diff <= atol + rtol * np.abs(want)
    rel_l2 = float(np.linalg.norm(diff) / max(np.linalg.norm(want.astype(np.float64)), 1e-30))
    return {
        "ok": finite and bool(within.all()),
        "finite": finite,
        "max_abs": float(diff.max()) if diff.size else 0.0,
        "rel_l2": rel_l2,
        "within": float(within.mean()) if diff.size else 1.0,
        "mismatch_bits": int((prng.bf16_bits(want) != prng.bf16_bits(got)).sum()),
    }
