"""The reference's PyTorch CPU implementation of the decoder_feedforward path, restated.

TEST/BASELINE INFRASTRUCTURE ONLY: bench.py's CPU-baseline leg (and `--impl reference`)
times this on the host cores; it is never the measured GPU path.

It builds the MLP exactly as scripts/generate_references.py:588-639 does: the real
transformers Gemma4 text MLP (gate/up/down nn.Linear in bf16, gelu_pytorch_tanh), each
projection wrapped to multiply its f32 output by the reciprocal NVFP4 global scale and
commit to bf16 (`GloballyScaled`, :588-602), with the dequantised NVFP4 weights
(codes * E4M3 block scale, exact in bf16, :622-626) installed, between the pre/post
feed-forward Gemma4RMSNorms, then the residual add and the per-layer scalar (:636-638).
"""

from __future__ import annotations

import os
import time

import torch

E2M1 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def dequant_nvfp4(packed: torch.Tensor, scale: torch.Tensor, rows: int, cols: int) -> torch.Tensor:
    p = packed.reshape(rows, cols // 2).to(torch.int64)
    codes = torch.stack([p & 0xF, p >> 4], dim=-1).reshape(rows, cols)
    vals = E2M1[codes & 7] * torch.where(codes >= 8, -1.0, 1.0)
    s = scale.reshape(rows, cols // 16).view(torch.float8_e4m3fn).float()
    return (vals * s.repeat_interleave(16, dim=-1)).to(torch.bfloat16)


class GloballyScaled(torch.nn.Module):
    def __init__(self, linear: torch.nn.Linear, scale: float):
        super().__init__()
        self.linear = linear
        self.scale = scale

    def forward(self, x):
        return (self.linear(x).float() * self.scale).to(x.dtype)


class ReferenceFeedforward:
    """decoder_feedforward on the CPU, built from config-1 style tensors (CPU torch)."""

    def __init__(self, m: dict, h: int = 3840, l: int = 15360):
        from transformers.models.gemma4 import configuration_gemma4 as C
        from transformers.models.gemma4 import modeling_gemma4 as M

        # the checkpoint's text config (generate_references.py:103-135)
        cfg = C.Gemma4TextConfig(hidden_size=h, intermediate_size=l, vocab_size=262144, num_attention_heads=16,
                                 num_key_value_heads=8, num_global_key_value_heads=1, head_dim=256,
                                 global_head_dim=512, num_hidden_layers=48, sliding_window=1024,
                                 rms_norm_eps=1e-6, hidden_activation="gelu_pytorch_tanh", attention_bias=False,
                                 attention_dropout=0.0, attention_k_eq_v=True, final_logit_softcapping=30.0,
                                 use_double_wide_mlp=False, enable_moe_block=False, num_kv_shared_layers=0,
                                 tie_word_embeddings=True,
                                 layer_types=["full_attention" if i % 6 == 5 else "sliding_attention"
                                              for i in range(48)],
                                 rope_parameters={
                                     "sliding_attention": {"rope_type": "default", "rope_theta": 10_000.0},
                                     "full_attention": {"rope_type": "proportional", "rope_theta": 1_000_000.0,
                                                        "partial_rotary_factor": 0.25}})
        torch.set_grad_enabled(False)
        mlp = M.Gemma4TextMLP(cfg, layer_idx=0).to(torch.bfloat16)
        for name, (r, c) in (("gate", (l, h)), ("up", (l, h)), ("down", (h, l))):
            w = dequant_nvfp4(m[f"{name}_weight_packed"].cpu(), m[f"{name}_weight_scale"].cpu(), r, c)
            getattr(mlp, f"{name}_proj").weight.copy_(w)
            setattr(mlp, f"{name}_proj", GloballyScaled(getattr(mlp, f"{name}_proj"),
                                                        float(m[f"{name}_global_scale"].cpu()[0])))
        self.mlp = mlp
        self.pre = M.Gemma4RMSNorm(h, eps=1e-6).to(torch.bfloat16)
        self.post = M.Gemma4RMSNorm(h, eps=1e-6).to(torch.bfloat16)
        self.pre.weight.copy_(m["pre_ff_rms_weight"].cpu())
        self.post.weight.copy_(m["post_ff_rms_weight"].cpu())
        self.layer_scalar = m["layer_scalar"].cpu()[0]

    def __call__(self, residual: torch.Tensor) -> torch.Tensor:
        hidden = self.post(self.mlp(self.pre(residual)))
        return ((residual + hidden).to(torch.bfloat16) * self.layer_scalar).to(torch.bfloat16)


def time_tokens(ref: ReferenceFeedforward, x: torch.Tensor, steps: int, warmup: int = 3,
                budget_s: float = 30.0):
    """Per-token CPU time of `ref`, the one timing method of both CPU legs of bench.py.

    `warmup` untimed tokens, then `steps` tokens timed one by one with perf_counter,
    stopping early only when `budget_s` seconds have passed (at least 3 tokens).
    Returns (median_s, tokens_timed, threads); all host threads are used."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    for _ in range(max(0, warmup)):
        ref(x)
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < steps and (len(times) < 3 or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        ref(x)
        times.append(time.perf_counter() - t0)
    times.sort()
    return times[len(times) // 2], len(times), threads
