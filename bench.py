#!/usr/bin/env python3
"""Benchmark of the hot path: decoder_feedforward (one decode token) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: one token through the NVFP4 GeGLU MLP block of Gemma-4-12B
(x ~ N(0,1) bf16, RMSNorm weights ~ N(0,0.1), gate/up [15360x3840] and down
[3840x15360] from N(0,0.02) quantized to NVFP4), seeded synthetic data.  A step is one
token through one layer's block; steps cycle through 4 layers' distinct weights
(4 x 99.6 MB > the 126 MB L2), so every step streams its weights from HBM.

N=1: `value` = device time per token (CUDA events on the launching stream).  N>1
(torchrun): tensor parallel, each rank holds 1/N of every layer (column-parallel
gate/up, row-parallel down) and the block ends in one all-reduce; `value` = the max over
ranks of the device time per token ("strong" scaling: the work per token is fixed).
`e2e` times the same op through the C ABI with the residual copied from pinned host
memory before and read back after every step, the host waiting for each step's result
(copy in, call and copy out replayed as one CUDA graph per step).  `--impl reference` times the reference's
PyTorch CPU path on this host's cores instead (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "furiosa-opt-gemma4-12b_b200"))

METRIC = "decoder_feedforward µs/token"
UNIT = "µs/token"
H, L = 3840, 15360
NLAYERS = 4
# algorithmic bytes of one token (TP1): NVFP4 codes + E4M3 block scales of gate/up/down,
# three f32 global scales, residual in/out, two norm weights, layer scalar
WEIGHT_BYTES = 3 * (L * H // 2) + 3 * (L * H // 16)
MLP_ARGS = ("residual", "pre_ff_rms_weight", "up_weight_packed", "gate_weight_packed", "down_weight_packed",
            "up_weight_scale", "gate_weight_scale", "down_weight_scale", "up_global_scale", "gate_global_scale",
            "down_global_scale", "post_ff_rms_weight", "layer_scalar")
ACT_BYTES = 12 + 2 * H * 2 + 2 * H * 2 + 16


def algorithmic_bytes(world: int) -> int:
    return WEIGHT_BYTES // world + ACT_BYTES


def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def profile_traffic(kernel: str) -> float | None:
    """DRAM bytes per launch of `kernel` from the committed ncu summary."""
    p = ROOT / "profiles" / "decoder_feedforward_traffic.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["dram_bytes_per_launch_by_kernel"][kernel])
        except Exception:
            return None
    return None


def mlp_kernel_name(choice: str, world: int, peer: bool = False) -> str:
    """Kernel decoder_feedforward runs with this bench choice (the library's own rule:
    the tcgen05 kernel on one GPU and on TP2 contexts that exchange over peer memory,
    else the streaming kernel)."""
    if choice == "auto":
        choice = "stream" if os.environ.get("G4B200_MLP_KERNEL") == "stream" else "tensor"
    tc = choice == "tensor" and (world == 1 or (peer and world == 2))
    return "mlp_tc_kernel" if tc else "mlp_kernel"


class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML while the timed region runs."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device: int, period_s: float = 0.005):
        self.samples, self.reasons, self.ok = [], set(), False
        self.period = period_s
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for b, name in self.REASONS.items():
                    if bits & b and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        self._stop.clear()
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self) -> dict:
        s = sorted(self.samples)
        return {"sm_mhz": s[len(s) // 2] if s else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(s)}


def make_layers(device: str, rank: int, world: int):
    import torch
    from g4formats import quant, tp

    layers = []
    for i in range(NLAYERS):
        m = quant.mlp_config1(seed=i, device=device)
        if world > 1:
            m = tp.shard_mlp(m, rank, world)
        layers.append(m)
    torch.cuda.synchronize()
    return layers


def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    import torch.distributed as dist

    import g4b200 as g4

    torch.cuda.set_device(local_rank)
    dev = f"cuda:{local_rank}"
    stream = torch.cuda.Stream(device=dev)
    tpinfo = None
    if world > 1:
        nid = [g4.Context.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(nid, src=0)
        tpinfo = (rank, world, nid[0])
    ctx = g4.Context(local_rank, stream=stream, tp=tpinfo)
    ctx.set_mlp_kernel(args.mlp_kernel)
    kernel = mlp_kernel_name(args.mlp_kernel, world, world > 1 and ctx.tp_peer_exchange)
    layers = make_layers(dev, rank, world)
    residual = layers[0]["residual"].clone()

    def step(i: int) -> None:
        m = dict(layers[i % NLAYERS])
        m["residual"] = residual
        g4.decoder_feedforward(ctx, **m)

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    stream.synchronize()
    if ctx.poll() != 0:
        raise RuntimeError("device status set during warm-up")
    if not torch.isfinite(residual.float()).all():
        raise RuntimeError("non-finite residual after warm-up")

    # ---------------------------------------------------------------- device-timed region
    # One round = NLAYERS steps (one per layer).  The round is captured once in a CUDA
    # graph and replayed, so Python's per-call overhead does not gate the device;
    # consecutive launches overlap through programmatic dependent launch, so the
    # per-step device time is the timed region / steps.  Steps beyond whole rounds are
    # launched directly (exactly `steps` launches in total).  Under TP the all-reduce
    # runs inside the kernel over peer memory, so the graph holds no NCCL call (on the
    # NCCL fallback it does, and is released before the process group).
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(NLAYERS):
            step(i)
    stream.synchronize()
    # replay the captured round a few times before timing: the first replays after capture
    # pay one-off costs (graph upload, instruction cache) that a long run never sees
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
    stream.synchronize()
    rounds, rem = divmod(args.steps, NLAYERS)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank)
    with sampler, torch.cuda.stream(stream):
        t0.record(stream)
        for _ in range(rounds):
            graph.replay()
        for i in range(rem):
            step(i)
        t1.record(stream)
        stream.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = t0.elapsed_time(t1)
    kernel_ms = total_ms / args.steps
    status = ctx.poll()
    del graph

    # ---------------------------------------------------------------- end to end (host buffers)
    # What a host program does per token: copy the residual in from pinned host memory,
    # call the C ABI entry point, copy the result back, wait.  The entry point is bound
    # to its device buffers once (Context.prepare) and the copies are plain
    # cudaMemcpyAsync calls on the op's stream, recorded with the call in a CUDA graph.
    from cuda.bindings import runtime as cudart

    host_in = torch.empty(H, dtype=torch.bfloat16, pin_memory=True)
    host_in.copy_(layers[0]["residual"].cpu())
    host_out = torch.empty(H, dtype=torch.bfloat16, pin_memory=True)
    calls = [ctx.prepare("g4_decoder_feedforward", residual, *[layers[j][k] for k in MLP_ARGS[1:]])
             for j in range(NLAYERS)]
    sh = stream.cuda_stream
    h2d, d2h = cudart.cudaMemcpyKind.cudaMemcpyHostToDevice, cudart.cudaMemcpyKind.cudaMemcpyDeviceToHost
    dres, hin, hout, nb = residual.data_ptr(), host_in.data_ptr(), host_out.data_ptr(), H * 2
    # One token's host work (copy in, call, copy out) is recorded once per layer as a CUDA
    # graph, so a step costs one launch call instead of three; the host still waits for
    # every token's result before it issues the next.
    e2e_graphs = []
    for j in range(NLAYERS):
        gj = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gj, stream=stream):
            cudart.cudaMemcpyAsync(dres, hin, nb, h2d, sh)
            calls[j]()
            cudart.cudaMemcpyAsync(hout, dres, nb, d2h, sh)
        e2e_graphs.append(gj)
    with torch.cuda.stream(stream):
        for j in range(2 * NLAYERS):
            e2e_graphs[j % NLAYERS].replay()
            cudart.cudaStreamSynchronize(sh)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = min(args.steps, 2000)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(e2e_steps):
            e2e_graphs[i % NLAYERS].replay()
            cudart.cudaStreamSynchronize(sh)
        e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    del e2e_graphs

    in_step = None
    if world == 1 and not args.no_ops:
        try:
            in_step = run_mlp_in_step(ctx, stream, layers, residual, dev)
        except Exception as e:  # the headline MLP line still prints
            in_step = {"error": f"{type(e).__name__}: {e}"}
    decode = None
    if not args.no_decode:
        try:
            decode = run_decode(args, ctx, stream, rank, world, dev)
        except Exception as e:  # the headline MLP line still prints
            decode = {"error": f"{type(e).__name__}: {e}"}
    ops_lines = None
    if world == 1 and not args.no_ops:
        try:
            ops_lines = run_ops(list(OP_BYTES), ctx, stream, dev)
        except Exception as e:  # the headline MLP line still prints
            ops_lines = [{"error": f"{type(e).__name__}: {e}"}]
    prefill = None
    if not args.no_prefill:
        try:
            prefill = run_prefill(args, ctx, stream, rank, world, dev)
        except Exception as e:  # the headline MLP line still prints
            prefill = {"error": f"{type(e).__name__}: {e}"}
    vals = torch.tensor([total_ms / args.steps, kernel_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms_per_step, kernel_ms, e2e_ms = vals.tolist()
    peer = ctx.tp_peer_exchange
    ctx.close()
    if rank != 0:
        return None

    peak, peak_kind = measured_peaks()
    achieved = algorithmic_bytes(world) / (kernel_ms * 1e-3) / 1e9
    traffic = profile_traffic(kernel) if world == 1 else None
    line = {
        "metric": METRIC, "value": round(ms_per_step * 1000.0, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "nvfp4 weights, bf16 act, f32 acc",
        "data": "synthetic (seeded N(0,1) x, N(0,0.1) norms, N(0,0.02) weights quantized to NVFP4)",
        "config": {"workload": "decoder_feedforward one token, BASELINE config 1 (H=3840, L=15360, NVFP4)",
                   "global_batch": 1, "seq_len": 1, "parallelism": f"tp{world}",
                   "layers_cycled": NLAYERS, "l2": f"inputs larger than L2 ({NLAYERS} layers x "
                   f"{WEIGHT_BYTES / 1e6:.1f} MB weights cycled per step)",
                   "kernel": kernel,
                   "launch": "CUDA graph of one round (one launch per layer) replayed; consecutive launches "
                             "overlap via programmatic dependent launch" + (
                                 "" if world == 1 else
                                 "; TP all-reduce inside the kernel over NVLink peer memory" if peer else
                                 "; TP all-reduce by NCCL, then a one-CTA epilogue kernel")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "traffic": traffic, "algorithmic_bytes_per_launch": algorithmic_bytes(world),
                     "kernel_us": round(kernel_ms * 1000.0, 3)},
        "e2e": {"value": round(e2e_ms * 1000.0, 3), "unit": UNIT, "h2d_bytes_per_step": H * 2,
                "d2h_bytes_per_step": H * 2,
                "launch": "per step: CUDA graph (H2D copy, C-ABI call, D2H copy) replayed, host waits"},
        "gpu_launches": args.steps * (1 if world == 1 or peer else 2),
        "clocks": sampler.summary(),
        "device_status": status,
    }
    if in_step is not None:
        line["mlp_in_step"] = in_step
    if decode is not None:
        line["decode"] = decode
    if prefill is not None:
        line["prefill"] = prefill
    if ops_lines is not None:
        line["ops"] = ops_lines
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args)
    return line


# Per-op lines (one GPU): the attention-side ops of the decode step and BASELINE configs 2
# and 3, each cycled over enough distinct weight or cache copies to exceed L2.
OP_BYTES = {
    "sliding_qkv": 31473664, "full_qkv": 33440768, "sliding_qkv_nvfp4": 17694720,
    "sliding_oproj": 15736320, "full_oproj": 31464960,
    "sliding_attn": 8388608, "full_attn_8192": 8192 * 512 * 2 * 2,
}


def run_mlp_in_step(ctx, stream, layers, residual, dev: str) -> dict:
    """The MLP's cost next to another kernel, as in a decode step: a CUDA graph of
    NLAYERS x (decoder_feedforward, then sliding_project_qkv reading its residual) against
    one of the NLAYERS projections alone; the difference per layer is what the MLP adds
    when its prologue overlaps a projection instead of another MLP's tail."""
    import torch

    import g4b200 as g4

    g = torch.Generator(device=dev).manual_seed(5)

    def bf(n, std=1.0):
        return (torch.randn(n, device=dev, generator=g) * std).to(torch.bfloat16)

    def f8(n):
        return torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g) & 0x77

    ones = torch.ones(H, dtype=torch.bfloat16, device=dev)
    qn = torch.ones(256, dtype=torch.bfloat16, device=dev)
    i32 = lambda v: torch.tensor([v], dtype=torch.int32, device=dev)  # noqa: E731
    kv_off, rope_off = i32((517 % 1024) * 8 * 256 * 2), i32(517 * 256 * 2)
    cs, sn = bf(32768 * 256, 0.5), bf(32768 * 256, 0.5)
    kc = torch.zeros(1024 * 8 * 256, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    q_out = torch.zeros(4096, dtype=torch.bfloat16, device=dev)
    qkv = [(f8(4096 * H), f8(2048 * H), f8(2048 * H), bf(4096, 0.01), bf(2048, 0.01), bf(2048, 0.01))
           for _ in range(NLAYERS)]

    def mlp(j):
        m = dict(layers[j])
        m["residual"] = residual
        g4.decoder_feedforward(ctx, **m)

    def proj(j):
        w = qkv[j]
        g4.sliding_project_qkv(ctx, residual, w[0], w[1], w[2], w[3], w[4], w[5], ones, qn, qn, kv_off, rope_off,
                               cs, sn, kc, vc, q_out)

    def timed(fn) -> float:
        with torch.cuda.stream(stream):
            for j in range(NLAYERS):
                fn(j)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for j in range(NLAYERS):
                fn(j)
        reps = 500
        with torch.cuda.stream(stream):
            for _ in range(3):
                graph.replay()
            stream.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
            stream.synchronize()
        del graph
        return e0.elapsed_time(e1) * 1000.0 / (reps * NLAYERS)

    pair = timed(lambda j: (mlp(j), proj(j)))
    alone = timed(proj)
    return {"value": round(pair - alone, 3), "unit": "µs/token", "pair_us": round(pair, 3),
            "projection_alone_us": round(alone, 3), "device_status": ctx.poll(),
            "how": "graph of decoder_feedforward + sliding_project_qkv per layer, minus the projections alone"}


def run_ops(names, ctx, stream, dev: str) -> list[dict]:
    """Times each op through its public wrapper: a CUDA graph of one round over `copies`
    distinct inputs (> 2x L2 of weights or caches) replayed, CUDA events on the stream."""
    import torch

    import g4b200 as g4

    g = torch.Generator(device=dev).manual_seed(2)

    def bf(n, std=1.0):
        return (torch.randn(n, device=dev, generator=g) * std).to(torch.bfloat16)

    def f8(n):  # finite E4M3 codes
        return torch.randint(0, 256, (n,), dtype=torch.uint8, device=dev, generator=g) & 0x77

    def ones_bf(n):
        return torch.ones(n, dtype=torch.bfloat16, device=dev)

    pos = 517
    i32 = lambda v: torch.tensor([v], dtype=torch.int32, device=dev)  # noqa: E731
    cos_s, sin_s = bf(32768 * 256, 0.5), bf(32768 * 256, 0.5)
    cos_f, sin_f = bf(32768 * 512, 0.5), bf(32768 * 512, 0.5)
    peak, peak_kind = measured_peaks()
    out = []
    for name in names:
        nbytes = OP_BYTES[name]
        copies = max(2, -(-320_000_000 // nbytes))
        calls = []
        if name in ("sliding_qkv", "full_qkv", "sliding_qkv_nvfp4"):
            full = name == "full_qkv"
            D = 512 if full else 256
            rows = (8192, 512, 0) if full else (4096, 2048, 2048)
            x, in_w, qn, kn = bf(H), ones_bf(H), ones_bf(D), ones_bf(D)
            kv_off = i32((pos % 512) * 512 * 2 if full else (pos % 1024) * 8 * 256 * 2)
            rope_off = i32(pos * D * 2)
            kc = torch.zeros((512 if full else 1024 * 8) * D, dtype=torch.bfloat16, device=dev)
            vc = torch.zeros_like(kc)
            q_out = torch.zeros(rows[0], dtype=torch.bfloat16, device=dev)
            cs, sn = (cos_f, sin_f) if full else (cos_s, sin_s)
            for _ in range(copies):
                if name == "sliding_qkv_nvfp4":
                    w = [f8(r * H // 2) for r in rows]
                    bs = [(torch.randint(0x30, 0x40, (r * H // 16,), dtype=torch.uint8, device=dev, generator=g))
                          for r in rows]
                    gs = [torch.full((1,), 1.0 / 64, dtype=torch.float32, device=dev) for _ in rows]
                    a = (x, *w, *bs, *gs, in_w, qn, kn, kv_off, rope_off, cs, sn, kc, vc, q_out)
                    calls.append(lambda a=a: g4.sliding_project_qkv_nvfp4(ctx, *a))
                elif full:
                    a = (x, f8(rows[0] * H), f8(rows[1] * H), bf(rows[0], 0.01), bf(rows[1], 0.01), in_w, qn, kn,
                         kv_off, rope_off, cs, sn, kc, vc, q_out)
                    calls.append(lambda a=a: g4.full_project_qkv(ctx, *a))
                else:
                    a = (x, f8(rows[0] * H), f8(rows[1] * H), f8(rows[2] * H), bf(rows[0], 0.01), bf(rows[1], 0.01),
                         bf(rows[2], 0.01), in_w, qn, kn, kv_off, rope_off, cs, sn, kc, vc, q_out)
                    calls.append(lambda a=a: g4.sliding_project_qkv(ctx, *a))
        elif name in ("sliding_oproj", "full_oproj"):
            full = name == "full_oproj"
            K = 8192 if full else 4096
            x, pw, res = bf(K), ones_bf(H), bf(H)
            rsum = torch.ones(16, dtype=torch.float32, device=dev)
            for _ in range(copies):
                w, sc = f8(H * K), bf(H, 0.001)
                if full:
                    calls.append(lambda w=w, sc=sc: g4.full_attention_output(ctx, x, rsum, pw, w, sc, res))
                else:
                    calls.append(lambda w=w, sc=sc: g4.sliding_attention_output(ctx, x, pw, w, sc, res))
        elif name == "sliding_attn":
            q, mask, o = bf(4096), torch.ones(1024, dtype=torch.float32, device=dev), bf(4096)
            for _ in range(copies):
                k, v = bf(1024 * 8 * 256), bf(1024 * 8 * 256)
                calls.append(lambda k=k, v=v: g4.sliding_attention(ctx, q, k, v, mask, o))
        else:  # full_attn_8192: the reference's page cache, 16 pages of [512, 512]
            q, o = bf(16 * 512), bf(16 * 512)
            rsum = torch.ones(16, dtype=torch.float32, device=dev)
            for _ in range(copies):
                kp, vp = bf(16 * 512 * 512), bf(16 * 512 * 512)
                ka = torch.tensor([kp.data_ptr() + i * 512 * 512 * 2 for i in range(16)], dtype=torch.int64,
                                  device=dev)
                va = torch.tensor([vp.data_ptr() + i * 512 * 512 * 2 for i in range(16)], dtype=torch.int64,
                                  device=dev)
                calls.append(lambda ka=ka, va=va, kp=kp, vp=vp: g4.full_attention_paged(ctx, q, ka, va, 16, 511,
                                                                                       rsum, o))
        with torch.cuda.stream(stream):
            for c in calls:
                c()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for c in calls:
                c()
        reps = max(3, 4000 // len(calls))
        with torch.cuda.stream(stream):
            for _ in range(3):
                graph.replay()
            stream.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
            stream.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / (reps * len(calls))
        del graph, calls
        achieved = nbytes / (us * 1e-6) / 1e9
        out.append({"op": name, "value": round(us, 3), "unit": "µs/call", "copies": copies,
                    "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                                 "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                                 "algorithmic_bytes_per_call": nbytes},
                    "launch": "CUDA graph of one round over the copies, replayed; consecutive calls overlap via "
                              "programmatic dependent launch"})
    status = ctx.poll()
    for o in out:
        o["device_status"] = status
    return out


def run_only(args, rank: int, world: int, local_rank: int) -> dict | None:
    """One sub-measurement on its own (--only decode|prefill), printed as its own line."""
    import torch

    import g4b200 as g4

    torch.cuda.set_device(local_rank)
    dev = f"cuda:{local_rank}"
    stream = torch.cuda.Stream(device=dev)
    tpinfo = None
    if world > 1:
        import torch.distributed as dist

        nid = [g4.Context.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(nid, src=0)
        tpinfo = (rank, world, nid[0])
    ctx = g4.Context(local_rank, stream=stream, tp=tpinfo)
    try:
        if args.only == "ops":
            if world > 1:
                return None
            names = list(OP_BYTES) if args.op == "all" else [args.op]
            out = {"ops": run_ops(names, ctx, stream, dev)}
        else:
            out = (run_decode if args.only == "decode" else run_prefill)(args, ctx, stream, rank, world, dev)
    finally:
        ctx.close()
    return out if rank == 0 else None


def _cpu_reference_tokens(steps: int, warmup: int, budget_s: float) -> tuple[float, int, int]:
    """The reference's PyTorch CPU decoder_feedforward (oracle/cpu_reference.py) on this
    host's cores, config-1 layer-0 inputs built by g4formats (library-free: the product
    library is not loaded).  Both CPU legs use this one method: `warmup` tokens, then up
    to `steps` tokens timed one by one, median."""
    sys.path.insert(0, str(ROOT))
    from g4formats import quant
    from oracle import cpu_reference

    m = quant.mlp_config1(seed=0, device="cpu")
    ref = cpu_reference.ReferenceFeedforward(m)
    return cpu_reference.time_tokens(ref, m["residual"], steps=steps, warmup=warmup, budget_s=budget_s)


# per-token algorithmic bytes of the whole-model decode step (TP1): every projection's
# weights once, the lm_head (the tied embedding table) once, and the KV rows attended
SLIDING_W = 31_473_664 + 15_736_320       # FP8 q/k/v + o-proj codes and row scales
FULL_W = 33_440_768 + 31_464_960
MLP_W = WEIGHT_BYTES + 12
LM_HEAD_W = 262144 * H * 2


def decode_bytes_per_token(n_layers: int, ctx_len: int, world: int) -> int:
    total = 0
    for i in range(n_layers):
        if i % 6 == 5:  # full (MQA) layer: the single K/V head is replicated on every rank
            total += FULL_W // world + MLP_W // world + min(ctx_len, 32768) * 512 * 2 * 2
        else:           # sliding: the rank's heads of the 1024-slot ring
            total += SLIDING_W // world + MLP_W // world + min(ctx_len, 1024) * 8 // world * 256 * 2 * 2
    return total + LM_HEAD_W // world


def run_decode(args, ctx, stream, rank: int, world: int, dev: str) -> dict:
    """BASELINE config 4 at batch 1: whole-model greedy decode (48 layers, 5 sliding : 1
    full) through the decode runtime, `decode_tokens` steps after a context of
    `decode_context` positions.  The KV caches of the context are filled with synthetic
    unit-RMS rows (the bytes each step reads do not depend on their values); each step is
    one replay of the captured step graph, position and token kept on the device."""
    import torch
    import torch.distributed as dist
    from cuda.bindings import runtime as cudart

    from g4b200 import runtime
    from g4formats import model as fm

    n_layers, ctx_len, n_new, warm = 48, args.decode_context, args.decode_tokens, 4
    t_build = time.time()
    m = fm.synthetic_model(n_layers, seed=7, device=dev, post_norm=0.05, layer_scalar=(1.0, 1.0))
    m = fm.shard_model(m, rank, world)
    rm = runtime.model_from_synthetic(m)
    ws = runtime.Workspace(ctx, rm, ctx_len + warm + n_new + 8)
    biggest = max(ws.kv_cache_ptrs(i)[2] for i in range(n_layers))
    fill = (fm.uniform("kv", 7, biggest // 2, dev) * 3.0 ** 0.5).to(torch.bfloat16)
    for i in range(n_layers):
        k, v, nb = ws.kv_cache_ptrs(i)
        for ptr in (k, v):
            cudart.cudaMemcpy(ptr, fill.data_ptr(), nb, cudart.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
    torch.cuda.synchronize()
    build_s = time.time() - t_build
    tok = 4242
    ws.begin([tok], ctx_len, warm + n_new)
    ws.steps(warm)  # the first captures the step graph
    stream.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(int(dev.split(":")[1]))
    with sampler:
        t0.record(stream)
        ws.steps(n_new)
        t1.record(stream)
        stream.synchronize()
    dev_ms = t0.elapsed_time(t1) / n_new
    toks = ws.tokens(warm + n_new)
    # end to end through the public call: prompt token from the host, the step graph
    # replayed per token, the generated ids copied back
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    gen = ws.generate([tok], n_new, start_pos=ctx_len)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / n_new
    vals = torch.tensor([dev_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    dev_ms, e2e_ms = vals.tolist()
    status = ctx.poll()
    ws.close()
    rm.close()
    del m
    peak, peak_kind = measured_peaks()
    nbytes = decode_bytes_per_token(n_layers, ctx_len + warm + n_new // 2, world)
    achieved = nbytes / (dev_ms * 1e-3) / 1e9
    return {
        "metric": "decode tokens/s", "value": round(1000.0 / dev_ms, 2), "unit": "tokens/s",
        "us_per_token": round(dev_ms * 1000.0, 2), "higher_is_better": True, "n_gpus": world,
        "config": {"workload": "whole-model greedy decode, BASELINE config 4 (48 layers: 40 sliding-1024 + 8 full, "
                               "5:1), batch 1", "context": ctx_len, "decode_steps": n_new, "warmup_steps": warm,
                   "parallelism": f"tp{world}", "weights": "FP8 attention (reference formats), NVFP4 MLP, bf16 "
                                                          "tied lm_head; seeded random init, 48 distinct layers",
                   "kv": "caches filled with synthetic rows for the context", "l2": "inputs larger than L2 "
                         f"({nbytes / 1e9:.2f} GB streamed per token)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                     "algorithmic_bytes_per_token": nbytes},
        "e2e": {"value": round(1000.0 / e2e_ms, 2), "unit": "tokens/s", "us_per_token": round(e2e_ms * 1000.0, 2),
                "h2d_bytes_per_step": round(4 / n_new, 3), "d2h_bytes_per_step": 4,
                "launch": "g4_generate_greedy: prompt id H2D, one step-graph replay per token, ids D2H"},
        "clocks": sampler.summary(), "device_status": status,
        "tokens_sample": toks[warm:warm + 8], "build_s": round(build_s, 1),
    }


PREFILL_ORDER = ("pre_ff_rms_weight", "up_weight_packed", "gate_weight_packed", "down_weight_packed",
                 "up_weight_scale", "gate_weight_scale", "down_weight_scale", "up_global_scale", "gate_global_scale",
                 "down_global_scale", "post_ff_rms_weight", "layer_scalar")


def run_prefill(args, ctx, stream, rank: int, world: int, dev: str) -> dict:
    """the MLP block of M tokens at once (g4_decoder_feedforward_prefill)
    on the block-scaled FP4 tensor cores, NVFP4 weights of config 1's distributions (seed
    4), x ~ N(0, 1) bf16.  Timed per call with CUDA events (max over ranks), for the
    default 2 activation pieces and for 1; e2e adds the residual's H2D copy from pinned
    memory and its D2H read-back to every call."""
    import torch
    import torch.distributed as dist

    import g4b200 as g4
    from g4formats import quant, tp

    M, reps = args.prefill_tokens, args.prefill_reps
    m = quant.mlp_config1(seed=4, device=dev)
    if world > 1:
        m = tp.shard_mlp(m, rank, world)
    w = [m[k] for k in PREFILL_ORDER]
    g = torch.Generator(device=dev).manual_seed(4)
    x0 = torch.randn(M, H, device=dev, generator=g).to(torch.bfloat16)
    flops = 2.0 * M * H * L * 3
    out = {}
    sampler = ClockSampler(int(dev.split(":")[1]))
    for pieces in (2, 1):
        ctx.set_prefill_pieces(pieces)
        r = x0.clone()
        with torch.cuda.stream(stream):
            for _ in range(3):
                g4.decoder_feedforward_prefill(ctx, r, *w)
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with sampler, torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                g4.decoder_feedforward_prefill(ctx, r, *w)
            e1.record(stream)
            stream.synchronize()
        ms = e0.elapsed_time(e1) / reps
        # end to end: the residual from pinned host memory and back, every call
        host_in = x0.cpu().pin_memory()
        host_out = torch.empty_like(host_in).pin_memory()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                r.copy_(host_in, non_blocking=True)
                g4.decoder_feedforward_prefill(ctx, r, *w)
                host_out.copy_(r, non_blocking=True)
            e1.record(stream)
            stream.synchronize()
        e2e_ms = e0.elapsed_time(e1) / reps
        vals = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        out[pieces] = vals.tolist()
    ctx.set_prefill_pieces(2)
    status = ctx.poll()
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    fp4_peak = 4.0 * bf16
    ms2, e2e2 = out[2]
    ms1, e2e1 = out[1]
    tf2, tf1 = flops / (ms2 * 1e-3) / 1e12, flops / (ms1 * 1e-3) / 1e12
    return {
        "metric": "prefill MLP TFLOP/s", "value": round(tf2, 1), "unit": "TFLOP/s", "higher_is_better": True,
        "n_gpus": world, "ms_per_call": round(ms2, 4), "dtype": "nvfp4 weights x nvfp4 activations (2 pieces), f32 acc",
        "config": {"workload": "batched prefill MLP, BASELINE config 5 (M=4096 tokens, H=3840, L=15360, NVFP4 "
                               "GeGLU block, tcgen05 kind::mxf4nvf4)", "tokens": M, "parallelism": f"tp{world}",
                   "activation_pieces": 2, "flops_per_call": flops,
                   "l2": "weights 99.5 MB + activations re-read from L2 across token tiles (one call per step)"},
        "roofline": {"bound": "tensor", "achieved": round(tf2, 1), "peak": round(fp4_peak, 1), "unit": "TFLOP/s",
                     "frac": round(tf2 / fp4_peak, 4),
                     "peak_kind": "4 x measured bf16 cuBLAS burst (MEASURED_PEAKS.json bf16_tflops): the FP4 MMA "
                                  "rate is 4x the bf16 rate; nominal dense FP4 9000",
                     "tensor_work_factor": 2},
        "one_piece": {"value": round(tf1, 1), "ms_per_call": round(ms1, 4), "frac": round(tf1 / fp4_peak, 4),
                      "e2e_tflops": round(flops / (e2e1 * 1e-3) / 1e12, 1)},
        "e2e": {"value": round(flops / (e2e2 * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "ms_per_call": round(e2e2, 4),
                "h2d_bytes_per_step": M * H * 2, "d2h_bytes_per_step": M * H * 2,
                "launch": "per call: pinned H2D copy of the residual, C-ABI call, D2H copy"},
        "gpu_launches_per_call": 5 + (1 if world == 8 else 0),
        "clocks": sampler.summary(), "device_status": status,
    }


def cpu_baseline(args) -> dict:
    """The reference's PyTorch CPU path (oracle port) on this host, bounded sample."""
    med, n, threads = _cpu_reference_tokens(args.steps, min(args.warmup, 5), args.cpu_budget)
    return {"value": round(med * 1e6, 1), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} tokens of decoder_feedforward (config 1, layer 0) after {min(args.warmup, 5)} warm-up, "
                      f"median, torch CPU bf16 GloballyScaled MLP as in scripts/generate_references.py:588-639"}


def run_reference(args, rank: int, world: int) -> dict | None:
    """`--impl reference`: the reference's CPU implementation of the path (the oracle
    port; the reference itself is Rust for an NPU and cannot run here), timed exactly
    like this arm's `cpu_baseline`.  Imports only g4formats and oracle/, never g4b200."""
    if rank != 0:
        return None
    med, n, threads = _cpu_reference_tokens(args.steps, min(args.warmup, 5), args.cpu_budget)
    v = round(med * 1e6, 1)
    return {
        "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": n, "warmup": args.warmup,
        "ms_per_step": round(med * 1e3, 4), "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 (dequantised NVFP4 weights), CPU", "data": "synthetic (same as ours)", "impl": "reference",
        "same_steps": n == args.steps,
        "config": {"workload": "decoder_feedforward one token, BASELINE config 1 (H=3840, L=15360, NVFP4)",
                   "global_batch": 1, "seq_len": 1, "parallelism": "cpu"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{n} tokens (median) after {min(args.warmup, 5)} warm-up, layer-0 weights, "
                                   f"torch CPU GloballyScaled MLP"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=30.0, help="seconds: cap of each CPU leg's timed tokens")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the whole-model decode measurement")
    ap.add_argument("--decode-context", type=int, default=4096)
    ap.add_argument("--decode-tokens", type=int, default=64)
    ap.add_argument("--no-prefill", action="store_true", help="skip the batched prefill MLP measurement")
    ap.add_argument("--prefill-tokens", type=int, default=4096)
    ap.add_argument("--prefill-reps", type=int, default=30)
    ap.add_argument("--only", choices=["decode", "prefill", "ops"], default=None,
                    help="run just the whole-model decode, the prefill or the per-op measurement")
    ap.add_argument("--op", choices=["all", *OP_BYTES], default="all", help="with --only ops: which op")
    ap.add_argument("--no-ops", action="store_true", help="skip the per-op lines")
    ap.add_argument("--mlp-kernel", choices=["auto", "stream", "tensor"], default="auto",
                    help="decoder_feedforward kernel: streaming (CUDA-core decode) or tcgen05 (one GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line:
            print(json.dumps(line), flush=True)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device(f"cuda:{local_rank}"))
    try:
        line = run_only(args, rank, world, local_rank) if args.only else run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    if line:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
