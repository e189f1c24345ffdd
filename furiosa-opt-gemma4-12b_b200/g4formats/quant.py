"""NVFP4 / FP8 weight formats of the checkpoint, and seeded synthetic workloads.

The reference only consumes pre-quantized checkpoints (src/host/load.rs:143-191): NVFP4
E2M1 codes packed [N, K/2] (low nibble = even element), one E4M3 scale per 16 K
elements [N, K/16], and one f32 per-tensor global scale whose RECIPROCAL the loader
hands to the kernels.  It ships no quantizer, so this module supplies one for the
benchmark's N(0, sigma) weight configurations, with the usual NVFP4 recipe:

    g      = 448 * 6 / max|W|                        (checkpoint `weight_global_scale`)
    s_b    = e4m3(max|W_b| / 6 * g)                  (block scale, round-to-nearest)
    code   = e2m1(W * g / s_b)                       (round-to-nearest-even, saturate 6)
    W     ~= code * s_b / g                          (kernels multiply by 1/g)

Everything runs in torch on the tensor's device (CPU or GPU) with the same bits on both:
every operation is an exactly rounded elementwise op or an exact reduction, and a
division by a constant is written as a tensor division (torch's CUDA kernels turn a
division by a Python number into a multiplication by its reciprocal, the CPU's do not).
"""

from __future__ import annotations

import torch

E2M1_GRID = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def e2m1_encode(x: torch.Tensor) -> torch.Tensor:
    """Nearest E2M1 code (ties to even mantissa), saturating at +/-6; returns uint8 codes."""
    a = x.abs()
    # thresholds between grid points; ties go to the even-mantissa neighbour
    idx = torch.zeros_like(a, dtype=torch.uint8)
    idx = torch.where(a > 0.25, 1, idx)
    idx = torch.where(a >= 0.75, 2, idx)
    idx = torch.where(a > 1.25, 3, idx)
    idx = torch.where(a >= 1.75, 4, idx)
    idx = torch.where(a > 2.5, 5, idx)
    idx = torch.where(a >= 3.5, 6, idx)
    idx = torch.where(a > 5.0, 7, idx).to(torch.uint8)
    sign = ((x < 0) & (idx > 0)).to(torch.uint8) << 3
    return idx | sign


def pack_e2m1(codes: torch.Tensor) -> torch.Tensor:
    """[N, K] codes -> [N, K/2] bytes, low nibble = even element."""
    c = codes.to(torch.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).contiguous()


def _div(x: torch.Tensor, c: float) -> torch.Tensor:
    """x / c, correctly rounded on the CPU and on a GPU alike."""
    return x / torch.full_like(x, c)


def quantize_nvfp4(w: torch.Tensor):
    """[N, K] float weights -> (packed u8 [N, K/2], block scales u8 [N, K/16], 1/g f32 [1])."""
    w = w.float()
    n, k = w.shape
    amax = w.abs().max().clamp_min(1e-30)
    g = torch.reciprocal(amax) * (448.0 * 6.0)  # what `2688.0 / amax` computes on either device
    blocks = w.view(n, k // 16, 16)
    bmax = blocks.abs().amax(dim=-1)
    s = (_div(bmax, 6.0) * g).clamp(max=448.0).to(torch.float8_e4m3fn)
    sf = s.float()
    scaled = torch.where(sf[..., None] > 0, blocks * g / sf[..., None].clamp_min(1e-30), torch.zeros_like(blocks))
    codes = e2m1_encode(scaled).view(n, k)
    recip = (1.0 / g).reshape(1).to(torch.float32)
    return pack_e2m1(codes), s.view(torch.uint8).contiguous(), recip.contiguous()


def quantize_fp8_rows(w: torch.Tensor):
    """[N, K] -> (e4m3 codes u8 [N, K], bf16 per-row scale [N]): the attention format
    (src/host/load.rs:22-56): W ~= code * scale_row."""
    w = w.float()
    rmax = w.abs().amax(dim=1).clamp_min(1e-30)
    scale = _div(rmax, 448.0).to(torch.bfloat16)
    codes = (w / scale.float()[:, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
    return codes.view(torch.uint8).contiguous(), scale.contiguous()


def bf16_normal(shape, std: float, gen: torch.Generator, device="cpu") -> torch.Tensor:
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


def mlp_config1(seed: int = 0, device="cpu", rows: int = 15360):
    """BASELINE config 1 inputs: x ~ N(0,1) bf16, RMSNorm weights ~ N(0, 0.1), gate/up
    [rows, 3840] and down [3840, rows] ~ N(0, 0.02) quantized to NVFP4; layer scalar 1.0
    (the reference model's default, scripts/gemma4.py:214)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    h = 3840
    out = {
        "residual": bf16_normal((h,), 1.0, gen, device),
        "pre_ff_rms_weight": bf16_normal((h,), 0.1, gen, device),
        "post_ff_rms_weight": bf16_normal((h,), 0.1, gen, device),
    }
    for name, shape in (("gate", (rows, h)), ("up", (rows, h)), ("down", (h, rows))):
        w = torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * 0.02
        p, s, g = quantize_nvfp4(w)
        out[f"{name}_weight_packed"] = p.reshape(-1)
        out[f"{name}_weight_scale"] = s.reshape(-1)
        out[f"{name}_global_scale"] = g
        del w
    out["layer_scalar"] = torch.ones(8, dtype=torch.bfloat16, device=device)
    return out
