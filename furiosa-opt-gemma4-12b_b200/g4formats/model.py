"""Seeded random-init weights of the whole text decoder, in the checkpoint's formats.

The reference loads a pre-quantized checkpoint (src/host/load.rs:357-386); none can be
downloaded here, so the decode runtime is driven by synthetic weights of the same
architecture, names, shapes and storage formats ("all projections
random-init"):

- every value comes from a stateless integer hash of (tensor name, element index), so
  the same call gives the same bits on the CPU and on a GPU (integer ops, then one
  f32 scale and the quantizers of `quant`, all exactly rounded elementwise ops);
- weights are uniform with standard deviation 0.02 (the embedding, and the projections
  before quantization: attention FP8 E4M3 with a bf16 row scale, src/host/load.rs:22-56;
  MLP NVFP4, load.rs:143-191); RMSNorm weights 1 + U(+-0.1) times a per-kind gain:
  q/k norms 0.25 (attention scores of standard deviation ~1 instead of ~16, so the
  softmax is not a near-argmax that flips on rounding noise), post-attention and
  post-feed-forward norms `post_norm` (small values keep a deep random model from
  amplifying rounding differences layer after layer), the final norm a random sign
  per element (the tied lm_head would otherwise mostly predict the input token back);
  layer scalars U[layer_scalar];
- layer i is a full-attention layer iff i % 6 == 5 (load.rs:369-376).  `distinct`
  layers are generated; layer i uses the weights of layer i % distinct (a 48-layer model
  whose 8 periods of 6 layers share weights keeps the CPU oracle's memory at 6 layers;
  every layer still has its own KV cache).

Tensor names and device formats are those of g4_model_set_tensor (include/g4.h).
"""

from __future__ import annotations

import torch

from . import quant

H, L, W = 3840, 15360, 262144
NS, GS, DS, QS, PS = 8, 2, 256, 4096, 2048
GF, DF, QF, PF = 16, 512, 8192, 512
PREFIX = "model.language_model.layers."
EMBED = "model.language_model.embed_tokens.weight"
FINAL_NORM = "model.language_model.norm.weight"
_M32 = 0xFFFFFFFF
_CHUNK = 1 << 24


def is_full(layer: int) -> bool:
    return layer % 6 == 5


def _fnv1a(s: str) -> int:
    h = 0x811C9DC5
    for b in s.encode():
        h = ((h ^ b) * 0x01000193) & _M32
    return h


def _hash32(x: torch.Tensor) -> torch.Tensor:
    """32-bit integer hash on int64 tensors holding values in [0, 2^32): every product
    stays below 2^63, so it is exact on any device."""
    x = x ^ (x >> 16)
    x = (x * 0x7FEB352D) & _M32
    x = x ^ (x >> 15)
    x = (x * 0x68E31DA5) & _M32
    return x ^ (x >> 16)


def uniform(name: str, seed: int, n: int, device) -> torch.Tensor:
    """n values U[-1, 1) (f32, multiples of 2^-23) from the hash of (seed, name, index)."""
    s = _fnv1a(f"{seed}:{name}")
    out = torch.empty(n, dtype=torch.float32, device=device)
    for c0 in range(0, n, _CHUNK):
        m = min(_CHUNK, n - c0)
        i = torch.arange(c0, c0 + m, dtype=torch.int64, device=device)
        h = _hash32(((i * 0x9E3779B1) + s) & _M32)
        h = _hash32(h ^ (s >> 1))
        u = (h >> 8).to(torch.float32) * (1.0 / (1 << 24))
        out[c0:c0 + m] = u * 2.0 - 1.0
    return out


def _u(name, seed, shape, std, device):
    n = 1
    for d in shape:
        n *= d
    return (uniform(name, seed, n, device) * (std * 3.0 ** 0.5)).reshape(shape)


def _norm_w(name, seed, n, device, gain: float = 1.0):
    return ((1.0 + 0.1 * uniform(name, seed, n, device)) * gain).to(torch.bfloat16)


def layer_tensors(layer: int, seed: int, device, post_norm: float = 1.0,
                  layer_scalar: tuple[float, float] = (0.4, 0.7)) -> dict[str, torch.Tensor]:
    """The tensors of one layer, checkpoint names relative to the layer prefix."""
    full = is_full(layer)
    key = f"L{layer}"
    out: dict[str, torch.Tensor] = {}
    for nm in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
               "post_feedforward_layernorm"):
        out[f"{nm}.weight"] = _norm_w(f"{key}.{nm}", seed, H, device, post_norm if nm.startswith("post") else 1.0)
    lo, hi = layer_scalar
    ls = (lo + hi) / 2 + (hi - lo) / 2 * uniform(f"{key}.layer_scalar", seed, 1, device)
    out["layer_scalar"] = ls.to(torch.bfloat16).repeat(8)
    q_rows, k_rows, d = (QF, PF, DF) if full else (QS, PS, DS)
    projs = [("q_proj", q_rows, H), ("k_proj", k_rows, H), ("o_proj", H, q_rows)]
    if not full:
        projs.insert(2, ("v_proj", k_rows, H))
    for nm, rows, cols in projs:
        w = _u(f"{key}.{nm}", seed, (rows, cols), 0.02, device)
        codes, scale = quant.quantize_fp8_rows(w)
        out[f"self_attn.{nm}.weight"] = codes.reshape(-1)
        out[f"self_attn.{nm}.weight_scale"] = scale.reshape(-1)
        del w
    out["self_attn.q_norm.weight"] = _norm_w(f"{key}.q_norm", seed, d, device, 0.25)
    out["self_attn.k_norm.weight"] = _norm_w(f"{key}.k_norm", seed, d, device, 0.25)
    for nm, shape in (("gate_proj", (L, H)), ("up_proj", (L, H)), ("down_proj", (H, L))):
        w = _u(f"{key}.{nm}", seed, shape, 0.02, device)
        p, s, g = quant.quantize_nvfp4(w)
        out[f"mlp.{nm}.weight_packed"] = p.reshape(-1)
        out[f"mlp.{nm}.weight_scale"] = s.reshape(-1)
        out[f"mlp.{nm}.weight_global_scale"] = g
        del w
    return out


def synthetic_model(n_layers: int, seed: int = 0, device="cpu", distinct: int | None = None,
                    post_norm: float = 1.0, layer_scalar: tuple[float, float] = (0.4, 0.7)) -> dict:
    """{"embed": ..., "final_norm": ..., "layers": [dict per distinct layer], "n_layers",
    "distinct"}: the whole decoder at tensor-parallel world 1."""
    distinct = n_layers if distinct is None else distinct
    if n_layers % distinct or (distinct < n_layers and distinct % 6):
        raise ValueError("distinct layers must divide n_layers and be a multiple of 6 when shared")
    embed = _u("embed", seed, (W, H), 0.02, device).to(torch.bfloat16)
    return {
        "embed": embed.reshape(-1),
        "final_norm": (_norm_w("final_norm", seed, H, device).float()
                       * torch.where(uniform("final_norm.sign", seed, H, device) < 0, -1.0, 1.0)).to(torch.bfloat16),
        "layers": [layer_tensors(i, seed, device, post_norm, layer_scalar) for i in range(distinct)],
        "n_layers": n_layers,
        "distinct": distinct,
    }


def checkpoint_names(model: dict) -> dict[str, torch.Tensor]:
    """Flat {checkpoint name: tensor} of every layer (shared weights appear once per layer)."""
    out = {EMBED: model["embed"], FINAL_NORM: model["final_norm"]}
    for i in range(model["n_layers"]):
        for k, t in model["layers"][i % model["distinct"]].items():
            out[f"{PREFIX}{i}.{k}"] = t
    return out


def _rows(t, rank, world, nrows):
    per = t.numel() // nrows
    n = nrows // world
    return t.reshape(-1)[rank * n * per:(rank + 1) * n * per].contiguous()


def _cols(t, rank, world, nrows, ncols):
    n = ncols // world
    return t.reshape(nrows, ncols)[:, rank * n:(rank + 1) * n].contiguous().reshape(-1)


def shard_layer(t: dict, layer: int, rank: int, world: int) -> dict:
    """The rank's shard of one layer: column-parallel q/k/v (heads) and gate/up, row-parallel
    o-proj and down; the full layers' single K head is replicated."""
    if world == 1:
        return t
    full = is_full(layer)
    q_rows, k_rows = (QF, PF) if full else (QS, PS)
    out = dict(t)
    out["self_attn.q_proj.weight"] = _rows(t["self_attn.q_proj.weight"], rank, world, q_rows)
    out["self_attn.q_proj.weight_scale"] = _rows(t["self_attn.q_proj.weight_scale"], rank, world, q_rows)
    if not full:
        for nm in ("k_proj", "v_proj"):
            out[f"self_attn.{nm}.weight"] = _rows(t[f"self_attn.{nm}.weight"], rank, world, k_rows)
            out[f"self_attn.{nm}.weight_scale"] = _rows(t[f"self_attn.{nm}.weight_scale"], rank, world, k_rows)
    out["self_attn.o_proj.weight"] = _cols(t["self_attn.o_proj.weight"], rank, world, H, q_rows)
    for nm in ("gate_proj", "up_proj"):
        out[f"mlp.{nm}.weight_packed"] = _rows(t[f"mlp.{nm}.weight_packed"], rank, world, L)
        out[f"mlp.{nm}.weight_scale"] = _rows(t[f"mlp.{nm}.weight_scale"], rank, world, L)
    out["mlp.down_proj.weight_packed"] = _cols(t["mlp.down_proj.weight_packed"], rank, world, H, L // 2)
    out["mlp.down_proj.weight_scale"] = _cols(t["mlp.down_proj.weight_scale"], rank, world, H, L // 16)
    return out


def shard_model(model: dict, rank: int, world: int) -> dict:
    if world == 1:
        return model
    out = dict(model)
    out["layers"] = [shard_layer(t, i, rank, world) for i, t in enumerate(model["layers"])]
    return out


def tensor_checksum(t: torch.Tensor) -> int:
    """Order-sensitive checksum of a tensor's bytes (the same on CPU and GPU), computed in
    chunks so a 2 GB table needs little extra memory."""
    b = t.contiguous().view(torch.uint8).reshape(-1)
    mod = (1 << 61) - 1
    total = 0
    for c0 in range(0, b.numel(), _CHUNK):
        c = b[c0:c0 + _CHUNK].to(torch.int64)
        idx = torch.arange(c0, c0 + c.numel(), dtype=torch.int64, device=b.device)
        total = (total + int((c * ((idx % 65521) + 1)).sum().item())) % mod
    return total
