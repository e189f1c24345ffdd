"""CPU oracle of the whole text decoder: one decode step after another, greedy.

TEST INFRASTRUCTURE ONLY (the checker for the decode runtime; never the measured path).

The step follows the reference host loop (src/host/runtime.rs:311-513): embed_token,
then per layer (full iff i % 6 == 5, src/host/load.rs:369-376)
  sliding: project_qkv -> K/V into ring slot pos % 1024 -> attention over the slots whose
           mask row min(pos, 1023) is 1 -> attention_output (+residual)
  full:    project_qkv -> K/V into row pos of the page array -> attention over rows 0..pos
           -> attention_output (+residual)
  decoder_feedforward,
then final_norm_and_logits and the first maximal logit (torch.argmax).  Each op uses the
rounding points of oracle/ops.py, i.e. of the reference's per-kernel generator
(scripts/generate_references.py): RMSNorm :80-94 of scripts/gemma4.py, FP8 projection
:312-321, q/k/v norms and RoPE :379-425 / :480-521, masked f32 softmax :324-330, attention
outputs :458-469 / :559-577, GloballyScaled MLP :588-639, lm_head and softcap :642-669,
embedding :347-368.  The RoPE tables are the kernel-side ones of rope_data
(src/host/runtime.rs:271-299: f32 angle pos / theta^(2i/dim), bf16 cos/sin).

The arithmetic is torch on the CPU in float32 with explicit bf16 rounding (the weights
are dequantised once: E4M3 codes for the FP8 projections, whose per-row scale is applied
after the f32 dot product, and E2M1 x E4M3 block scale for the MLP, exact in bf16).
"""

from __future__ import annotations

import numpy as np
import torch

H, L, W = 3840, 15360, 262144
NS, GS, DS, TS = 8, 2, 256, 1024
GF, DF = 16, 512
EPS = 1e-6
EMBED_SCALE = 61.967734

_E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def rb(x: torch.Tensor) -> torch.Tensor:
    """Round float32 to bf16 (nearest even) and back."""
    return x.to(torch.bfloat16).to(torch.float32)


def rms_norm(x: torch.Tensor, w: torch.Tensor | None) -> torch.Tensor:
    """oracle.ops.rms_norm over the last axis: f32 squares summed in f64, 1/sqrt, bf16."""
    ms = (x * x).double().sum(-1, keepdim=True).float()
    ms = ms / float(x.shape[-1]) + EPS
    r = 1.0 / torch.sqrt(ms)
    y = x * r
    if w is not None:
        y = y * w
    return rb(y)


def e4m3(codes: torch.Tensor) -> torch.Tensor:
    return codes.view(torch.float8_e4m3fn).to(torch.float32)


def dequant_nvfp4(packed: torch.Tensor, scale: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    p = packed.reshape(rows, cols // 2).to(torch.int64)
    codes = torch.stack([p & 0xF, p >> 4], dim=-1).reshape(rows, cols)
    vals = _E2M1[codes & 7] * torch.where(codes >= 8, -1.0, 1.0)
    return vals * e4m3(scale.reshape(rows, cols // 16)).repeat_interleave(16, dim=-1)


def rope_tables(dim: int, theta: float, rotated_dim: int, pos: int):
    """cos and (upstream-convention) sin of one position from rope_data's f32 math."""
    half, rhalf = dim // 2, rotated_dim // 2
    i = np.arange(half, dtype=np.float32)
    inv = np.power(np.float32(theta), (np.float32(2) * i) / np.float32(dim), dtype=np.float32)
    f = (np.float32(pos) / inv).astype(np.float32)
    c = np.where(i < rhalf, np.cos(f, dtype=np.float32), np.float32(1.0))
    s = np.where(i < rhalf, np.sin(f, dtype=np.float32), np.float32(0.0))
    c = torch.from_numpy(np.concatenate([c, c]).astype(np.float32))
    s = torch.from_numpy(np.concatenate([s, s]).astype(np.float32))
    return rb(c), rb(s)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return rb(rb(x * cos) + rb(rot * sin))


def softmax_attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """oracle.ops.masked_softmax_attention over the given rows: q [h, D], k/v [T, D]."""
    s = (q.double() @ k.double().T).float()
    m = s.max(dim=-1, keepdim=True).values
    e = torch.exp(s - m)
    p = e / e.double().sum(-1, keepdim=True).float()
    return rb((p.double() @ v.double()).float())


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    inner = 0.7978845608028654 * (x + 0.044715 * (x * x * x))
    return 0.5 * x * (1.0 + torch.tanh(inner))


class Layer:
    """One layer's weights, dequantised for the CPU."""

    def __init__(self, t: dict, full: bool):
        f = lambda k: t[k].to(torch.float32)  # noqa: E731
        self.full = full
        self.in_w, self.post_attn_w = f("input_layernorm.weight"), f("post_attention_layernorm.weight")
        self.pre_ff_w, self.post_ff_w = f("pre_feedforward_layernorm.weight"), f("post_feedforward_layernorm.weight")
        self.layer_scalar = float(t["layer_scalar"][0].float())
        q_rows, k_rows, d = (8192, 512, DF) if full else (4096, 2048, DS)
        self.d = d
        self.wq = e4m3(t["self_attn.q_proj.weight"]).reshape(q_rows, H)
        self.sq = f("self_attn.q_proj.weight_scale")
        self.wk = e4m3(t["self_attn.k_proj.weight"]).reshape(k_rows, H)
        self.sk = f("self_attn.k_proj.weight_scale")
        if not full:
            self.wv = e4m3(t["self_attn.v_proj.weight"]).reshape(k_rows, H)
            self.sv = f("self_attn.v_proj.weight_scale")
        self.wo = e4m3(t["self_attn.o_proj.weight"]).reshape(H, q_rows)
        self.so = f("self_attn.o_proj.weight_scale")
        self.qn, self.kn = f("self_attn.q_norm.weight"), f("self_attn.k_norm.weight")
        mats = {}
        for nm, (r, c) in (("gate", (L, H)), ("up", (L, H)), ("down", (H, L))):
            mats[nm] = dequant_nvfp4(t[f"mlp.{nm}_proj.weight_packed"], t[f"mlp.{nm}_proj.weight_scale"], r, c)
            setattr(self, f"g_{nm}", float(t[f"mlp.{nm}_proj.weight_global_scale"][0]))
        self.wg, self.wu, self.wd = mats["gate"], mats["up"], mats["down"]


def proj(w: torch.Tensor, x: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """FP8 projection: bf16((x @ codes.T) * scale)."""
    return rb((w @ x) * scale)


def gscaled(w: torch.Tensor, x: torch.Tensor, g: float) -> torch.Tensor:
    """GloballyScaled NVFP4 projection: bf16(bf16(x @ W.T) * g)."""
    return rb(rb(w @ x) * torch.tensor(g, dtype=torch.float32))


class Decoder:
    """The decode loop state: weights (shared periods allowed), KV caches, position."""

    def __init__(self, model: dict):
        torch.set_grad_enabled(False)
        self.n_layers = model["n_layers"]
        self.distinct = model["distinct"]
        self.layers = [Layer(t, i % 6 == 5) for i, t in enumerate(model["layers"])]
        self.table = model["embed"].reshape(W, H)
        self.final_w = model["final_norm"].to(torch.float32)
        self.kc, self.vc = [], []
        for i in range(self.n_layers):
            self.kc.append({})
            self.vc.append({})
        self._lm = None

    def lm_head(self) -> torch.Tensor:
        if self._lm is None:
            self._lm = self.table.to(torch.float32)
        return self._lm

    def step(self, token: int, pos: int, logits: bool = True):
        """One position; returns (x after the last layer, logits or None)."""
        x = rb(self.table[token].to(torch.float32) * rb(torch.tensor(EMBED_SCALE, dtype=torch.float32)))
        cs = rope_tables(DS, 10000.0, DS, pos)
        cf = rope_tables(DF, 1_000_000.0, 128, pos)
        for i in range(self.n_layers):
            ly = self.layers[i % self.distinct]
            h = rms_norm(x, ly.in_w)
            if not ly.full:
                q = rope(rms_norm(proj(ly.wq, h, ly.sq).reshape(-1, DS), ly.qn), *cs)
                k = rope(rms_norm(proj(ly.wk, h, ly.sk).reshape(-1, DS), ly.kn), *cs)
                v = rms_norm(proj(ly.wv, h, ly.sv).reshape(-1, DS), None)
                slot = pos % TS
                self.kc[i][slot], self.vc[i][slot] = k, v
                lo = max(0, pos - (TS - 1))
                slots = [p % TS for p in range(lo, pos + 1)]
                K = torch.stack([self.kc[i][s] for s in slots])  # [T, NS, DS]
                V = torch.stack([self.vc[i][s] for s in slots])
                qh = q.reshape(NS, GS, DS)
                out = torch.stack([softmax_attend(qh[n], K[:, n], V[:, n]) for n in range(NS)])
            else:
                q = rope(rms_norm(proj(ly.wq, h, ly.sq).reshape(-1, DF), ly.qn), *cf)
                k_raw = proj(ly.wk, h, ly.sk)
                k = rope(rms_norm(k_raw, ly.kn), *cf)
                v = rms_norm(k_raw, None)
                self.kc[i][pos], self.vc[i][pos] = k, v
                K = torch.stack([self.kc[i][p] for p in range(pos + 1)])
                V = torch.stack([self.vc[i][p] for p in range(pos + 1)])
                out = softmax_attend(q, K, V)
            o = proj(ly.wo, out.reshape(-1), ly.so)
            x = rb(x + rms_norm(o, ly.post_attn_w))
            # decoder_feedforward
            hm = rms_norm(x, ly.pre_ff_w)
            gate = gscaled(ly.wg, hm, ly.g_gate)
            up = gscaled(ly.wu, hm, ly.g_up)
            act = rb(rb(gelu_tanh(gate)) * up)
            down = gscaled(ly.wd, act, ly.g_down)
            x = rb(rb(x + rms_norm(down, ly.post_ff_w)) * ly.layer_scalar)
        if not logits:
            return x, None
        normed = rms_norm(x, self.final_w)
        lg = rb(self.lm_head() @ normed)
        lg = rb(torch.tanh(lg / 30.0) * 30.0)
        return x, lg

    def generate(self, prompt: list[int], max_new: int, start_pos: int = 0, on_step=None) -> list[int]:
        """Greedy: prompt positions start_pos.. one per step, then max_new predictions."""
        out: list[int] = []
        pos = start_pos
        for j, tok in enumerate(prompt):
            last = j == len(prompt) - 1
            x, lg = self.step(tok, pos, logits=last)
            if on_step:
                on_step(pos, x, lg)
            pos += 1
        nxt = int(torch.argmax(lg))
        out.append(nxt)
        while len(out) < max_new:
            x, lg = self.step(out[-1], pos)
            if on_step:
                on_step(pos, x, lg)
            pos += 1
            out.append(int(torch.argmax(lg)))
        return out
