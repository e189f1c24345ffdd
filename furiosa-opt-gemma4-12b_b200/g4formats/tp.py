"""Tensor-parallel sharding of the hot-path weights (the layout the C ABI expects when a
context is rank r of N, see g4_ctx_init_tp in include/g4.h).

Column-parallel (rows split): gate/up [L, H], q/k/v [heads*D, H], lm_head [W, H].
Row-parallel (K split): down [H, L], o-proj [H, heads*D].  NVFP4 K-slices stay aligned
to the 16-element scale blocks.  The full-attention single K/V head is replicated.
The reference runs on one chip and has no sharding (src/lib.rs:17); its checkpoint
layout (src/host/load.rs) is what gets cut.
"""

from __future__ import annotations


def rows(t, rank: int, world: int, nrows: int):
    """Rows [rank*nrows/world, (rank+1)*nrows/world) of a row-major [nrows, ...] buffer."""
    per = t.numel() // nrows
    n = nrows // world
    return t.reshape(-1)[rank * n * per:(rank + 1) * n * per].contiguous()


def cols(t, rank: int, world: int, nrows: int, ncols: int):
    """Column slice of a row-major [nrows, ncols] buffer, made contiguous."""
    n = ncols // world
    return t.reshape(nrows, ncols)[:, rank * n:(rank + 1) * n].contiguous().reshape(-1)


def shard_mlp(m: dict, rank: int, world: int, h: int = 3840, l: int = 15360) -> dict:
    """decoder_feedforward arguments of rank `rank` (gate/up rows, down K-slice)."""
    out = dict(m)
    for name in ("gate", "up"):
        out[f"{name}_weight_packed"] = rows(m[f"{name}_weight_packed"], rank, world, l)
        out[f"{name}_weight_scale"] = rows(m[f"{name}_weight_scale"], rank, world, l)
    out["down_weight_packed"] = cols(m["down_weight_packed"], rank, world, h, l // 2)
    out["down_weight_scale"] = cols(m["down_weight_scale"], rank, world, h, l // 16)
    return out
