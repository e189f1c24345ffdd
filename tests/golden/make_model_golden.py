#!/usr/bin/env python3
"""Golden greedy-decode fixtures for the decode runtime, pinned to the reference's model.

For each case (a seeded synthetic model of g4formats.model, a seeded prompt):
  1. the CPU oracle (oracle/model.py, one decode step after another, as the reference's
     host loop src/host/runtime.rs:311-513 runs the kernels) prefills the prompt and
     greedily decodes `new` tokens;
  2. with the reference checkout given, the reference's own PyTorch model
     (scripts/gemma4.py: Gemma4ForCausalLM, its layers, norms, RoPE tables, SDPA
     attention, tied lm_head and softcap) runs ONE teacher-forced forward over prompt +
     generated tokens, with the synthetic weights installed.  Its projections are wrapped
     the way the reference's kernel generator wraps them (scripts/generate_references.py:
     FP8 `scaled_projection` :312-321 and NVFP4 `GloballyScaled` :588-602), so both sides
     compute the same per-op math and differ only in composition;  the script records
     how many of the oracle's greedy tokens are the reference model's argmax too and the
     largest logit difference, and fails if they disagree beyond near-ties;
  3. it writes tests/golden/model_golden.npz: per case the model's tensor checksums (so
     a GPU test can prove it rebuilt the same weights), the prompt, the oracle's greedy
     tokens, the top-8 logits (values, indices) of every generated step, and the hidden
     state after the last layer (bf16 bits) at every 16th generated step and the last.

Usage:  python tests/golden/make_model_golden.py [<reference checkout>]
        (or G4B200_REFERENCE_DIR=...; without it the reference check is skipped)
"""

from __future__ import annotations

import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "furiosa-opt-gemma4-12b_b200"))

from g4formats import model as fm  # noqa: E402
from oracle import model as om  # noqa: E402

OUT = HERE / "model_golden.npz"
# name: (layers, distinct layers, model seed, prompt length, new tokens, post-norm gain x 1000,
#        layer scalar range x 1000)
CASES = {
    # crosses page 512, page 1024 and the sliding ring's wrap at 1024
    "six_layers_long": (6, 6, 1, 1100, 64, 1000, 400, 700),
    # 48 layers, 8 periods sharing 6 layers' weights (each layer its own KV cache)
    "full_depth": (48, 6, 2, 64, 64, 50, 1000, 1000),
}


def build(spec, device="cpu"):
    n_layers, distinct, seed, _, _, post, lo, hi = spec
    return fm.synthetic_model(n_layers, seed=seed, device=device, distinct=distinct, post_norm=post / 1000,
                              layer_scalar=(lo / 1000, hi / 1000))


def prompt_tokens(seed: int, n: int) -> list[int]:
    u = fm.uniform("prompt", seed, n, "cpu")
    return [int(x) for x in ((u + 1.0) * 0.5 * fm.W).clamp(0, fm.W - 1).to(torch.int64)]


def checksums(m: dict) -> dict[str, int]:
    out = {"embed": fm.tensor_checksum(m["embed"]), "final_norm": fm.tensor_checksum(m["final_norm"])}
    for i, lt in enumerate(m["layers"]):
        for k, t in lt.items():
            out[f"{i}.{k}"] = fm.tensor_checksum(t)
    return out


def reference_check(ref_dir: Path, m: dict, tokens: list[int], n_prompt: int, gen: list[int]) -> dict:
    sys.path.insert(0, str(ref_dir / "scripts"))
    import gemma4 as g  # noqa: E402  (the reference's own model file)

    torch.set_grad_enabled(False)
    cfg = g.Gemma4Config(num_hidden_layers=m["n_layers"])
    model = g.Gemma4ForCausalLM(cfg).to(torch.bfloat16).eval()

    class Fp8Linear(torch.nn.Module):  # scaled_projection (generate_references.py:312-321)
        def __init__(self, codes, scale):
            super().__init__()
            self.codes, self.scale = codes, scale

        def forward(self, x):
            return ((x.float() @ self.codes.T) * self.scale).to(torch.bfloat16)

    class GloballyScaled(torch.nn.Module):  # generate_references.py:588-602
        def __init__(self, w, s):
            super().__init__()
            self.w, self.s = w, s

        def forward(self, x):
            return (torch.nn.functional.linear(x, self.w).float() * self.s).to(torch.bfloat16)

    shared = []
    for i, lt in enumerate(m["layers"]):
        ly = om.Layer(lt, fm.is_full(i))
        mods = {"q_proj": Fp8Linear(ly.wq, ly.sq), "k_proj": Fp8Linear(ly.wk, ly.sk),
                "o_proj": Fp8Linear(ly.wo, ly.so)}
        if not ly.full:
            mods["v_proj"] = Fp8Linear(ly.wv, ly.sv)
        mlp = {"gate_proj": GloballyScaled(ly.wg.to(torch.bfloat16), ly.g_gate),
               "up_proj": GloballyScaled(ly.wu.to(torch.bfloat16), ly.g_up),
               "down_proj": GloballyScaled(ly.wd.to(torch.bfloat16), ly.g_down)}
        shared.append((lt, mods, mlp, ly))
    for i, layer in enumerate(model.layers):
        lt, mods, mlp, ly = shared[i % m["distinct"]]
        for k, v in mods.items():
            setattr(layer.self_attn, k, v)
        for k, v in mlp.items():
            setattr(layer.mlp, k, v)
        layer.self_attn.q_norm.weight.copy_(lt["self_attn.q_norm.weight"])
        layer.self_attn.k_norm.weight.copy_(lt["self_attn.k_norm.weight"])
        for nm in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                   "post_feedforward_layernorm"):
            getattr(layer, nm).weight.copy_(lt[f"{nm}.weight"])
        layer.layer_scalar.fill_(float(lt["layer_scalar"][0].float()))
    model.embed_tokens.weight.copy_(m["embed"].reshape(fm.W, fm.H))
    model.norm.weight.copy_(m["final_norm"])

    # Gemma4ForCausalLM.forward (scripts/gemma4.py:241-268), logits only where compared
    ids = torch.tensor([tokens], dtype=torch.int64)
    T = ids.shape[1]
    x = model.embed_tokens(ids)
    cs = {"sliding_attention": g.precompute_rope(cfg.head_dim, T, cfg.local_rope_theta, 1.0, x.device, x.dtype),
          "full_attention": g.precompute_rope(cfg.global_head_dim, T, cfg.global_rope_theta,
                                              cfg.global_partial_rotary_factor, x.device, x.dtype)}
    for i, layer in enumerate(model.layers):
        x = layer(x, *cs[cfg.layer_types[i]])
    x = model.norm(x[:, n_prompt - 1:])
    logits = model.lm_head(x).float()
    logits = torch.tanh(logits / cfg.final_logit_softcapping) * cfg.final_logit_softcapping
    ref_tokens = logits[0].argmax(-1).tolist()
    agree = sum(int(a == b) for a, b in zip(ref_tokens, gen))
    # near-tie: where they differ, the reference's logits of both tokens within 1/4
    gaps = []
    for j, (a, b) in enumerate(zip(ref_tokens, gen)):
        if a != b:
            gaps.append(float(logits[0, j, a] - logits[0, j, b]))
    return {"agree": agree, "total": len(gen), "disagree_gaps": gaps, "ref_tokens": ref_tokens}


def run_case(name: str, spec, ref_dir: Path | None) -> dict:
    n_layers, distinct, seed, n_prompt, n_new = spec[:5]
    t0 = time.time()
    m = build(spec)
    print(f"[{name}] model built in {time.time() - t0:.0f}s", flush=True)
    sums = checksums(m)
    prompt = prompt_tokens(seed, n_prompt)
    dec = om.Decoder(m)
    tops, hid, hid_pos = [], [], []
    keep = {n_prompt - 1 + j for j in range(0, n_new, 16)} | {n_prompt + n_new - 2}

    def on_step(pos, x, lg):
        if lg is not None:
            v, i = torch.topk(lg, 8)
            tops.append(np.concatenate([v.numpy().astype(np.float64), i.numpy().astype(np.float64)]))
        if pos in keep:
            hid.append(x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))
            hid_pos.append(pos)

    t0 = time.time()
    gen = dec.generate(prompt, n_new, on_step=on_step)
    print(f"[{name}] oracle decode in {time.time() - t0:.0f}s: {gen[:8]}...", flush=True)
    out = {"spec": np.array(spec, dtype=np.int64), "prompt": np.array(prompt, dtype=np.int32),
           "tokens": np.array(gen, dtype=np.int32), "top8": np.array(tops, dtype=np.float64),
           "hidden": np.array(hid), "hidden_pos": np.array(hid_pos, dtype=np.int32),
           "checksum_names": np.array(list(sums)), "checksums": np.array(list(sums.values()), dtype=np.int64)}
    if ref_dir is not None:
        t0 = time.time()
        r = reference_check(ref_dir, m, prompt + gen[:-1], n_prompt, gen)
        print(f"[{name}] reference model agrees on {r['agree']}/{r['total']} greedy tokens "
              f"({time.time() - t0:.0f}s); gaps where not: {r['disagree_gaps']}", flush=True)
        out["ref_agree"] = np.array([r["agree"], r["total"]], dtype=np.int64)
        out["ref_tokens"] = np.array(r["ref_tokens"], dtype=np.int32)
        out["ref_gaps"] = np.array(r["disagree_gaps"], dtype=np.float64)
        if any(abs(gp) > 0.25 for gp in r["disagree_gaps"]):
            raise SystemExit(f"[{name}] oracle and reference model disagree beyond a near-tie")
    return out


def main() -> None:
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("G4B200_REFERENCE_DIR")
    ref_dir = Path(ref) if ref else None
    only = os.environ.get("G4B200_GOLDEN_CASES")
    entries = {}
    if OUT.exists():
        old = np.load(OUT)
        entries = {k: old[k] for k in old.files}
    for name, spec in CASES.items():
        if only and name not in only.split(","):
            continue
        for k, v in run_case(name, spec, ref_dir).items():
            entries[f"{name}.{k}"] = v
        np.savez_compressed(OUT, **entries)
        print(f"wrote {OUT}", flush=True)


if __name__ == "__main__":
    main()
