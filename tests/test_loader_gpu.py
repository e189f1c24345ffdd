"""g4_model_load_safetensors on a B200: a checkpoint written in the reference's layout
(src/host/load.rs) loads to the same device weights, and so the same greedy tokens and
bit-identical hidden states, as the same model registered tensor by tensor."""

import pytest
import torch

import g4b200 as g4
from g4b200 import runtime
from g4formats import checkpoint
from g4formats import model as fm

pytestmark = pytest.mark.gpu


def test_loaded_checkpoint_decodes_like_the_registered_model(tmp_path):
    m = fm.synthetic_model(6, seed=11, device="cuda", post_norm=0.05, layer_scalar=(1.0, 1.0))
    path = tmp_path / "model.safetensors"
    checkpoint.save(m, str(path))
    assert runtime.check_checkpoint(path, 6) == (True, "")
    # the loader stores 1 / (checkpoint value): register the same f32 reciprocal directly
    for lt in m["layers"]:
        for nm in ("up_proj", "gate_proj", "down_proj"):
            g = lt[f"mlp.{nm}.weight_global_scale"]
            lt[f"mlp.{nm}.weight_global_scale"] = 1.0 / (1.0 / g.float())
    ctx = g4.Context(0, stream=torch.cuda.Stream())
    direct = runtime.model_from_synthetic(m)
    loaded = runtime.load_checkpoint(ctx, path, 6)
    prompt = [int(x) for x in ((fm.uniform("p", 11, 24, "cpu") + 1) * 0.5 * (fm.W - 1))]
    outs = []
    for model in (direct, loaded):
        ws = runtime.Workspace(ctx, model, 64)
        toks = ws.generate(prompt, 16)
        outs.append((toks, ws.hidden(), ws.logits()))
        ws.close()
    assert outs[0][0] == outs[1][0]
    assert torch.equal(outs[0][1], outs[1][1]) and torch.equal(outs[0][2], outs[1][2])
    assert ctx.poll() == 0
    loaded.close()
    direct.close()
    ctx.close()


def test_loader_rejects_a_bad_checkpoint_with_the_tensor_name(tmp_path):
    p = tmp_path / "bad.safetensors"
    checkpoint.sparse_skeleton(str(p), 1, global_scale=float("inf"))
    ctx = g4.Context(0)
    with pytest.raises(g4.G4Error) as e:
        runtime.load_checkpoint(ctx, p, 1)
    assert "weight_global_scale" in str(e.value)
    ctx.close()
