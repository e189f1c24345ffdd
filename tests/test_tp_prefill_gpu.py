"""Tensor-parallel batched prefill (g4_decoder_feedforward_prefill) and sampling
(g4_sample_top_k_top_p) on 2, 4 or 8 GPUs, ranks as child processes.  Each rank holds its gate/up rows and its down k-slice (8-way:
120-byte scale rows, which the library re-lays out for TMA), quantises its own slice of
h, and the ranks' f32 down sums are all-reduced over NCCL before the tail.

  * every rank ends with the same residual, bit for bit;
  * rank 0's result matches oracle/ops.py:prefill_feedforward with the same tensor-parallel
    split (h quantised per rank slice) within the single-GPU prefill tolerance;
  * sampling over vocab slices: every rank draws the same id, the oracle's on the whole
    vocabulary (the ranks' top-k candidates are all-gathered).

NVLS is off (NCCL_NVLS_ENABLE=0).  Skipped with fewer GPUs than ranks.
"""

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

ORDER = ("pre_ff_rms_weight", "up_weight_packed", "gate_weight_packed", "down_weight_packed", "up_weight_scale",
         "gate_weight_scale", "down_weight_scale", "up_global_scale", "gate_global_scale", "down_global_scale",
         "post_ff_rms_weight", "layer_scalar")
N_TOK = 130
PREFILL_REL_L2 = 2e-2


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank: int, world: int, port: int, q) -> None:
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import numpy as np
    import torch.distributed as dist

    import g4b200 as g4
    from g4formats import quant, tp

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    res = {}
    try:
        m = quant.mlp_config1(seed=4, device="cuda")
        sh = tp.shard_mlp(m, rank, world)
        nid = [g4.Context.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(nid, src=0)
        ctx = g4.Context(rank, tp=(rank, world, nid[0]))
        g = torch.Generator(device="cuda").manual_seed(44)
        r0 = torch.randn(N_TOK, 3840, device="cuda", generator=g).to(torch.bfloat16)
        r = r0.clone()
        g4.decoder_feedforward_prefill(ctx, r, *[sh[k] for k in ORDER])
        torch.cuda.synchronize()
        assert ctx.poll() == 0
        outs = [torch.empty_like(r) for _ in range(world)]
        dist.all_gather(outs, r)
        res["identical"] = all(torch.equal(outs[0], o) for o in outs)
        if rank == 0:
            from oracle import ops

            L, H = ops.L, ops.H
            mc = {k: v.cpu() for k, v in m.items()}
            deq = {n: ops.nvfp4_dequant(mc[f"{n}_weight_packed"].numpy().reshape(rr, kk // 2),
                                        mc[f"{n}_weight_scale"].numpy().reshape(rr, kk // 16))
                   for n, rr, kk in (("gate", L, H), ("up", L, H), ("down", H, L))}
            f = lambda t: t.float().cpu().numpy()  # noqa: E731
            want = ops.prefill_feedforward(f(r0), f(mc["pre_ff_rms_weight"]), f(mc["post_ff_rms_weight"]),
                                           deq["up"], deq["gate"], deq["down"], np.float32(mc["up_global_scale"][0]),
                                           np.float32(mc["gate_global_scale"][0]),
                                           np.float32(mc["down_global_scale"][0]), f(mc["layer_scalar"])[0],
                                           pieces=2, world=world)
            base = f(r0)
            a, b = want - base, f(r) - base
            res["rel_l2"] = float(np.linalg.norm(a - b) / np.linalg.norm(a))
        # sampling: the rank's vocab slice, the same draw everywhere
        from oracle import prng
        from oracle import sampling as smp

        W = 262144
        xs = np.tanh(np.random.default_rng(9).standard_normal(W).astype(np.float32) * 0.1) * 30.0
        bits = prng.bf16_bits(xs.astype(np.float32)).astype(np.uint16)
        sl = W // world
        mine = torch.from_numpy(bits[rank * sl:(rank + 1) * sl].view(np.int16).copy()).view(torch.bfloat16).cuda()
        u = torch.zeros(1, dtype=torch.float32, device="cuda")
        out = torch.zeros(1, dtype=torch.int32, device="cuda")
        picks, want = [], []
        for uu in (0.0, 0.3, 0.77, 0.99):
            u.fill_(uu)
            g4.sample_top_k_top_p(ctx, mine, 1.0, 64, 0.95, [5, 7], u, out)
            torch.cuda.synchronize()
            picks.append(int(out.item()))
            want.append(smp.sample(bits, 1.0, 64, 0.95, [5, 7], uu))
        t = torch.tensor(picks, dtype=torch.int32, device="cuda")
        ts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(ts, t)
        res["sample_identical"] = all(torch.equal(ts[0], x) for x in ts)
        res["sample_picks"] = picks
        res["sample_want"] = want
        dist.barrier()
        ctx.close()
    finally:
        if rank == 0:
            q.put(res)
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_prefill(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=900)
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    print(f"TP{world} prefill: ranks identical {res['identical']}, contribution rel-L2 {res['rel_l2']:.3e}")
    assert res["identical"], res
    assert res["rel_l2"] <= PREFILL_REL_L2, res
    assert res["sample_identical"], res
    assert res["sample_picks"] == res["sample_want"], res
