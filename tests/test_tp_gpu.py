"""Tensor parallelism on 2 (or 4) GPUs, ranks as child processes: the MLP and o-proj
kernels all-reduce their partial outputs themselves over NVLink peer memory.

  * rank results are bit-identical (every rank sums the partials in rank order) and
    match the single-GPU launch on the full weights within the MLP parity tolerance;
  * 300 launches in a row (the exchange alternates buffer halves per launch) stay
    identical across ranks;
  * the NCCL fallback (G4B200_TP_EXCHANGE=nccl on every rank) gives the same result;
  * a peer that never launches makes the waiting rank's bounded wait give up with
    DEV_ERR_TIMEOUT_PEER after the context's wait budget, and the GPU stays usable.

NVLS is off (NCCL_NVLS_ENABLE=0) and the kernels use plain peer loads and stores.
Skipped with fewer than 2 GPUs.
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
MLP_ATOL, MLP_REL_L2 = 0.02, 1e-2
H, QS = 3840, 4096


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _ctx(g4, dist, rank, world):
    nid = [g4.Context.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(nid, src=0)
    return g4.Context(rank, tp=(rank, world, nid[0]))


def _gather_identical(dist, t) -> bool:
    outs = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(outs, t)
    return all(torch.equal(outs[0], o) for o in outs)


def _ffn(g4, ctx, r, sh, n):
    for _ in range(n):
        g4.decoder_feedforward(ctx, r, *[sh[k] for k in ORDER])


def _rank(rank: int, world: int, port: int, q) -> None:
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ.pop("G4B200_TP_EXCHANGE", None)
    import numpy as np
    import torch.distributed as dist

    import g4b200 as g4
    from g4formats import quant, tp

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    res = {}
    try:
        m = quant.mlp_config1(seed=7, device="cuda")
        sh = tp.shard_mlp(m, rank, world)
        ctx = _ctx(g4, dist, rank, world)
        res["peer_path"] = ctx.tp_peer_exchange

        # three layers in a row (same weights), residual carried
        r = m["residual"].clone()
        _ffn(g4, ctx, r, sh, 3)
        torch.cuda.synchronize()
        assert ctx.poll() == 0
        res["mlp_identical"] = _gather_identical(dist, r)
        if rank == 0:
            c1 = g4.Context(0)
            r1 = m["residual"].clone()
            _ffn(g4, c1, r1, m, 3)
            torch.cuda.synchronize()
            a, b = r1.float().cpu().numpy(), r.float().cpu().numpy()
            d = np.abs(a - b)
            res["mlp_max_abs"] = float(d.max())
            res["mlp_rel_l2"] = float(np.linalg.norm(d) / np.linalg.norm(a))
            c1.close()

        # many launches back to back: the exchange's buffer halves alternate per launch
        dist.barrier()  # rank 0's single-GPU check above must not eat the peers' wait budget
        rs = m["residual"].clone()
        _ffn(g4, ctx, rs, sh, 300)
        torch.cuda.synchronize()
        assert ctx.poll() == 0
        res["stress_identical"] = _gather_identical(dist, rs)
        res["stress_finite"] = bool(torch.isfinite(rs.float()).all())

        # o-proj (sliding, FP8): rank r holds heads [r*QS/N, ...) of x and Wo's K-slice
        dist.barrier()
        g = torch.Generator(device="cuda").manual_seed(5)
        xo = torch.randn(QS, device="cuda", generator=g).to(torch.bfloat16)
        wo = torch.randint(0, 256, (H * QS,), dtype=torch.uint8, device="cuda", generator=g) & 0x77
        so = (torch.randn(H, device="cuda", generator=g) * 0.01).to(torch.bfloat16)
        pw = (torch.randn(H, device="cuda", generator=g) * 0.1).to(torch.bfloat16)
        res0 = torch.randn(H, device="cuda", generator=g).to(torch.bfloat16)
        ro = res0.clone()
        g4.sliding_attention_output(ctx, tp.rows(xo, rank, world, QS), pw, tp.cols(wo, rank, world, H, QS), so, ro)
        torch.cuda.synchronize()
        assert ctx.poll() == 0
        res["oproj_identical"] = _gather_identical(dist, ro)
        if rank == 0:
            c1 = g4.Context(0)
            r1 = res0.clone()
            g4.sliding_attention_output(c1, xo, pw, wo, so, r1)
            torch.cuda.synchronize()
            a, b = r1.float().cpu().numpy(), ro.float().cpu().numpy()
            d = np.abs(a - b)
            res["oproj_max_abs"] = float(d.max())
            res["oproj_rel_l2"] = float(np.linalg.norm(d) / np.linalg.norm(a))
            c1.close()

        # the NCCL fallback on every rank: same sums, tail in its own kernel
        os.environ["G4B200_TP_EXCHANGE"] = "nccl"
        cn = _ctx(g4, dist, rank, world)
        os.environ.pop("G4B200_TP_EXCHANGE")
        res["nccl_path"] = not cn.tp_peer_exchange
        rn = m["residual"].clone()
        _ffn(g4, cn, rn, sh, 3)
        torch.cuda.synchronize()
        assert cn.poll() == 0
        dn = (rn.float() - r.float()).abs()
        res["nccl_max_abs"] = float(dn.max())
        cn.close()

        # a peer that never launches: rank 0's wait gives up after 100 ms
        dist.barrier()
        if rank == 0:
            ctx.set_wait_budget(100_000)
            rt = m["residual"].clone()
            _ffn(g4, ctx, rt, sh, 1)
            torch.cuda.synchronize()
            try:
                ctx.poll()
                res["timeout"] = "no error"
            except g4.G4Error as e:
                res["timeout"] = str(e)
            x = torch.ones(1024, device="cuda")
            res["usable_after"] = float((x * 2).sum().item()) == 2048.0
        dist.barrier()  # the peer keeps its buffer mapped until rank 0's kernel is done
        ctx.close()
        dist.barrier()
    finally:
        if rank == 0:
            q.put(res)
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_peer_allreduce(world):
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
        res = q.get(timeout=600)
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    assert res["peer_path"] and res["nccl_path"], res
    assert res["mlp_identical"] and res["stress_identical"] and res["oproj_identical"], res
    assert res["stress_finite"], res
    assert res["mlp_max_abs"] <= MLP_ATOL and res["mlp_rel_l2"] <= MLP_REL_L2, res
    assert res["oproj_max_abs"] <= 0.1 and res["oproj_rel_l2"] <= 1e-2, res
    assert res["nccl_max_abs"] <= MLP_ATOL, res
    assert "G4_ERR" in res["timeout"] or "timed out" in res["timeout"], res
    assert res["usable_after"], res
