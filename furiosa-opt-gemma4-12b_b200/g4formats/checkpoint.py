"""Writes a model of g4formats.model as a safetensors checkpoint in the reference's layout.

The layout is the one src/host/load.rs reads (:89-386): checkpoint names, BF16 norms,
F8_E4M3 projections with BF16 row scales [N, 1], NVFP4 U8 codes [N, K/2], F8_E4M3 block
scales [N, K/16], a scalar F32 global scale that is the checkpoint value (the loader
takes its reciprocal), and a BF16 [1] layer scalar.  Used to exercise the library's
loader (g4_model_load_safetensors) on the same weights a test registers directly.

`sparse_skeleton` writes a file with the right header whose tensor bytes are left as
holes (zeros), except the global scales: enough for the loader's checks without
gigabytes of data.
"""

from __future__ import annotations

import json
import struct

import torch

from . import model as fm

H, L, W = fm.H, fm.L, fm.W


def _layer_entries(i: int, lt: dict | None):
    """(name, dtype, shape, tensor-or-None) of one layer in checkpoint form."""
    p = f"{fm.PREFIX}{i}."
    full = fm.is_full(i)
    q, k, d = (fm.QF, fm.PF, fm.DF) if full else (fm.QS, fm.PS, fm.DS)
    g = (lambda n: lt[n]) if lt is not None else (lambda n: None)  # noqa: E731
    out = []
    for nm in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
               "post_feedforward_layernorm"):
        out.append((p + nm + ".weight", "BF16", [H], g(nm + ".weight")))
    out.append((p + "layer_scalar", "BF16", [1], None if lt is None else lt["layer_scalar"][:1]))
    projs = [("q_proj", q, H), ("k_proj", k, H), ("o_proj", H, q)]
    if not full:
        projs.insert(2, ("v_proj", k, H))
    for nm, r, c in projs:
        out.append((p + f"self_attn.{nm}.weight", "F8_E4M3", [r, c], g(f"self_attn.{nm}.weight")))
        out.append((p + f"self_attn.{nm}.weight_scale", "BF16", [r, 1], g(f"self_attn.{nm}.weight_scale")))
    out.append((p + "self_attn.q_norm.weight", "BF16", [d], g("self_attn.q_norm.weight")))
    out.append((p + "self_attn.k_norm.weight", "BF16", [d], g("self_attn.k_norm.weight")))
    for nm, r, c in (("up_proj", L, H), ("gate_proj", L, H), ("down_proj", H, L)):
        out.append((p + f"mlp.{nm}.weight_packed", "U8", [r, c // 2], g(f"mlp.{nm}.weight_packed")))
        out.append((p + f"mlp.{nm}.weight_scale", "F8_E4M3", [r, c // 16], g(f"mlp.{nm}.weight_scale")))
        gs = None if lt is None else (1.0 / lt[f"mlp.{nm}.weight_global_scale"].float().cpu()).reshape([])
        out.append((p + f"mlp.{nm}.weight_global_scale", "F32", [], gs))
    return out


def _entries(model: dict | None, n_layers: int):
    ents = [(fm.EMBED, "BF16", [W, H], None if model is None else model["embed"]),
            (fm.FINAL_NORM, "BF16", [H], None if model is None else model["final_norm"])]
    for i in range(n_layers):
        lt = None if model is None else model["layers"][i % model["distinct"]]
        ents += _layer_entries(i, lt)
    return ents


_SIZE = {"BF16": 2, "F8_E4M3": 1, "U8": 1, "F32": 4}


def _header(ents) -> tuple[bytes, list[int]]:
    hdr, offs, off = {}, [], 0
    for name, dt, shape, _ in ents:
        n = _SIZE[dt]
        for s in shape:
            n *= s
        hdr[name] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + n]}
        offs.append(off)
        off += n
    hdr["__metadata__"] = {"format": "pt"}
    raw = json.dumps(hdr).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    return raw, offs


def save(model: dict, path: str, n_layers: int | None = None) -> None:
    """Every tensor of `model` (first n_layers layers) as a safetensors file."""
    n_layers = model["n_layers"] if n_layers is None else n_layers
    ents = _entries(model, n_layers)
    raw, _ = _header(ents)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for _, dt, _, t in ents:
            t = t.detach().contiguous().cpu()
            if dt == "F32":
                t = t.to(torch.float32)
            f.write(t.reshape(-1).view(torch.uint8).numpy().tobytes())


def sparse_skeleton(path: str, n_layers: int, global_scale: float = 9600.0, edit=None) -> None:
    """A checkpoint of the right header with zero-filled (sparse) tensor data, except the
    global scales.  `edit(name, record)` returns the header record to write for a tensor
    (changed or not), or None to leave the tensor out."""
    ents = _entries(None, n_layers)
    raw, offs = _header(ents)
    if edit is not None:
        hdr = json.loads(raw)
        hdr = {k: (v if k == "__metadata__" else edit(k, v)) for k, v in hdr.items()}
        hdr = {k: v for k, v in hdr.items() if v is not None}
        raw = json.dumps(hdr).encode()
        raw += b" " * ((8 - len(raw) % 8) % 8)
    total = 8 + len(raw) + sum(_SIZE[dt] * _prod(shape) for _, dt, shape, _ in ents)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        base = 8 + len(raw)
        for (name, dt, _, _), off in zip(ents, offs):
            if dt == "F32":
                f.seek(base + off)
                f.write(struct.pack("<f", global_scale))
        f.truncate(total)


def _prod(shape) -> int:
    n = 1
    for s in shape:
        n *= s
    return n
