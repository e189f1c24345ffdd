"""Tensor-parallel host logic on CPU: two `gloo` ranks shard one NVFP4 GeGLU MLP the way
the library expects a rank's weights (g4formats.tp.shard_mlp: gate/up rows, down K-slice
on 16-element scale-block boundaries), each computes its part with the oracle, and the
all-reduced partial down projection must equal the unsharded one.  Small shapes: the
sharding code takes the model dimensions as arguments."""

import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from g4formats import quant, tp
from oracle import ops

HS, LS = 256, 512  # hidden / intermediate sizes of the test MLP


def _mlp(seed: int) -> dict:
    gen = torch.Generator().manual_seed(seed)
    out = {"x": quant.bf16_normal((HS,), 1.0, gen, "cpu")}
    for name, shape in (("gate", (LS, HS)), ("up", (LS, HS)), ("down", (HS, LS))):
        w = torch.randn(shape, generator=gen) * 0.02
        p, s, g = quant.quantize_nvfp4(w)
        out[f"{name}_weight_packed"] = p.reshape(-1)
        out[f"{name}_weight_scale"] = s.reshape(-1)
        out[f"{name}_global_scale"] = g
    return out


def _np(t: torch.Tensor) -> np.ndarray:
    return t.numpy() if t.dtype != torch.bfloat16 else t.float().numpy()


def _partial_down(m: dict, rows: int) -> np.ndarray:
    """f32 down-projection sums (before the global scale) of the rows this dict holds."""
    x = _np(m["x"]).astype(np.float32)
    deq = lambda n, r, k: ops.nvfp4_dequant(_np(m[f"{n}_weight_packed"]).reshape(r, k // 2),  # noqa: E731
                                            _np(m[f"{n}_weight_scale"]).reshape(r, k // 16))
    gate = ops.globally_scaled_linear(x, deq("gate", rows, HS), np.float32(m["gate_global_scale"][0]))
    up = ops.globally_scaled_linear(x, deq("up", rows, HS), np.float32(m["up_global_scale"][0]))
    h = ops.rb(ops.rb(ops.gelu_tanh(gate)) * up)
    wd = deq("down", HS, rows)
    return (wd.astype(np.float32) @ h.astype(np.float32)).astype(np.float32)


def _rank(rank: int, world: int, port: int, q) -> None:
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        m = _mlp(seed=3)
        sh = tp.shard_mlp(m, rank, world, h=HS, l=LS)
        part = torch.from_numpy(_partial_down(sh, LS // world))
        dist.all_reduce(part)
        # every rank's shard pieces, gathered, must tile the full tensors exactly
        pieces = {k: [torch.empty_like(sh[k]) for _ in range(world)]
                  for k in ("gate_weight_packed", "up_weight_scale", "down_weight_packed", "down_weight_scale")}
        for k, lst in pieces.items():
            dist.all_gather(lst, sh[k])
        if rank == 0:
            full = _partial_down(m, LS)
            gate_rows = torch.cat(pieces["gate_weight_packed"])
            up_s_rows = torch.cat(pieces["up_weight_scale"])
            down_cols = torch.cat([p.reshape(HS, -1) for p in pieces["down_weight_packed"]], dim=1).reshape(-1)
            down_scols = torch.cat([p.reshape(HS, -1) for p in pieces["down_weight_scale"]], dim=1).reshape(-1)
            q.put({
                "max_abs": float(np.abs(part.numpy() - full).max()),
                "scale": float(np.abs(full).max()),
                "tiles": bool(torch.equal(gate_rows, m["gate_weight_packed"]) and
                              torch.equal(up_s_rows, m["up_weight_scale"]) and
                              torch.equal(down_cols, m["down_weight_packed"]) and
                              torch.equal(down_scols, m["down_weight_scale"])),
            })
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_two_rank_sharded_mlp_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res["tiles"], "the shards do not tile the full weights"
    # f32 sums over a different grouping: equal to rounding of a few ulps of the largest term
    assert res["max_abs"] <= 1e-5 * max(res["scale"], 1.0), res


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_sizes(world):
    m = _mlp(seed=1)
    sh = tp.shard_mlp(m, world - 1, world, h=HS, l=LS)
    assert sh["gate_weight_packed"].numel() == LS // world * HS // 2
    assert sh["up_weight_scale"].numel() == LS // world * HS // 16
    assert sh["down_weight_packed"].numel() == HS * LS // world // 2
    assert sh["down_weight_scale"].numel() == HS * LS // world // 16
