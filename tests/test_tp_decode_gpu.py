"""The decode runtime under tensor parallelism (2 or 4 GPUs, ranks as child processes):
each rank holds its shard of the six-layer golden model (column-parallel q/k/v heads and
gate/up rows, row-parallel o-proj and down, vocab-parallel lm_head), the MLP and o-proj
all-reduce over NVLink peer memory inside their kernels, and the greedy token is the
maximum of the ranks' (value, index) candidates gathered with NCCL.

Teacher-forced on the oracle's tokens, as test_decode_gpu.py does on one GPU: every
rank must make the same pick at every step and hold a bit-identical hidden state, the
picks must be the oracle's or near-ties, and the hidden state within the same bound.
NVLS is off (NCCL_NVLS_ENABLE=0).  Skipped with fewer GPUs than ranks.
"""

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden" / "model_golden.npz"
CASE = "six_layers_long"
NEAR_TIE = 0.25
HIDDEN_REL_L2 = 3e-2


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank: int, world: int, port: int, q) -> None:
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, str(Path(__file__).parent / "golden"))
    import torch.distributed as dist

    import g4b200 as g4
    import make_model_golden as mg
    from g4b200 import runtime
    from g4formats import model as fm

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    res = {}
    try:
        gold = np.load(GOLDEN)
        spec = tuple(int(x) for x in gold[f"{CASE}.spec"])
        m = fm.shard_model(mg.build(spec, device=f"cuda:{rank}"), rank, world)
        nid = [g4.Context.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(nid, src=0)
        ctx = g4.Context(rank, stream=torch.cuda.Stream(), tp=(rank, world, nid[0]))
        res["peer_path"] = ctx.tp_peer_exchange
        rm = runtime.model_from_synthetic(m)
        prompt = gold[f"{CASE}.prompt"].tolist()
        tokens = gold[f"{CASE}.tokens"].tolist()
        seq = prompt + tokens[:-1]
        ws = runtime.Workspace(ctx, rm, len(seq) + 16)
        last = int(gold[f"{CASE}.hidden_pos"][-1])
        ws.begin(seq, 0, 0)
        ws.steps(last + 1)
        hid = ws.hidden()
        ws.steps(len(seq) - last - 1)
        preds = ws.predictions(len(seq))
        assert ctx.poll() == 0
        outs = [torch.empty_like(hid) for _ in range(world)]
        dist.all_gather(outs, hid)
        res["hidden_identical"] = all(torch.equal(outs[0], o) for o in outs)
        pt = torch.tensor(preds, dtype=torch.int32, device=f"cuda:{rank}")
        po = [torch.empty_like(pt) for _ in range(world)]
        dist.all_gather(po, pt)
        res["preds_identical"] = all(torch.equal(po[0], o) for o in po)
        if rank == 0:
            want = torch.from_numpy(gold[f"{CASE}.hidden"][-1].view(np.int16)).view(torch.bfloat16).float()
            res["hidden_rel_l2"] = float((hid.float().cpu() - want).norm() / want.norm())
            n_prompt = spec[3]
            top8 = gold[f"{CASE}.top8"]
            same, worst = 0, 0.0
            for j, want_tok in enumerate(tokens):
                got = preds[n_prompt - 1 + j]
                if got == want_tok:
                    same += 1
                    continue
                idx = top8[j, 8:].astype(np.int64)
                hit = np.nonzero(idx == got)[0]
                gap = float(top8[j, 0] - top8[j, hit[0]]) if hit.size else float("inf")
                worst = max(worst, gap)
            res["same"], res["worst_gap"], res["n"] = same, worst, len(tokens)
        ws.close()
        rm.close()
        dist.barrier()
        ctx.close()
        dist.barrier()
    finally:
        if rank == 0:
            q.put(res)
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_decode_matches_oracle(world):
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
    print(f"TP{world} decode:", res)
    for p in procs:
        assert p.exitcode == 0
    assert res["peer_path"], res
    assert res["hidden_identical"] and res["preds_identical"], res
    assert res["hidden_rel_l2"] <= HIDDEN_REL_L2, res
    assert res["worst_gap"] <= NEAR_TIE, res
