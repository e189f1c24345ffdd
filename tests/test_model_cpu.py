"""The decode runtime's host side without a GPU: the weight-set registry of g4_model
(checkpoint names, layer pattern, argument checks), the synthetic weight generator and
its tensor-parallel cut, and the whole-model oracle's building blocks."""

import ctypes

import numpy as np
import pytest
import torch

import g4b200
from g4b200 import runtime
from g4formats import model as fm
from oracle import model as om

FAKE = 0x7F0000000000  # a 16-byte aligned address that is never dereferenced


def test_layer_pattern_is_five_sliding_then_one_full():
    # src/host/load.rs:369-376: layer % 6 == 5 is a full-attention layer
    assert [runtime.layer_is_full(i) for i in range(12)] == [i % 6 == 5 for i in range(12)]
    assert sum(runtime.layer_is_full(i) for i in range(48)) == 8


def test_model_registry_accepts_checkpoint_names_and_rejects_others():
    m = runtime.Model(6)
    lib = g4b200.LIB
    ok = [fm.EMBED, fm.FINAL_NORM, "model.language_model.layers.0.self_attn.v_proj.weight",
          "model.language_model.layers.5.self_attn.q_proj.weight", "model.language_model.layers.3.layer_scalar",
          "model.language_model.layers.2.mlp.down_proj.weight_global_scale"]
    for n in ok:
        assert lib.g4_model_set_tensor(m.handle, n.encode(), FAKE, 16) == 0, n
    bad = ["model.language_model.layers.5.self_attn.v_proj.weight",   # full layers have no v_proj
           "model.language_model.layers.6.input_layernorm.weight",    # beyond n_layers
           "model.language_model.layers.x.input_layernorm.weight",
           "model.vision_embedder.patch_ln1.weight", "lm_head.weight"]
    for n in bad:
        assert lib.g4_model_set_tensor(m.handle, n.encode(), FAKE, 16) == 1, n
    assert lib.g4_model_set_tensor(m.handle, fm.EMBED.encode(), FAKE + 8, 16) == 1  # misaligned
    assert b"16-byte" in lib.g4_model_last_error(m.handle)
    m.close()
    h = ctypes.c_void_p()
    assert lib.g4_model_create(0, ctypes.byref(h)) == 1
    assert lib.g4_model_create(49, ctypes.byref(h)) == 1


def test_uniform_generator_is_deterministic_and_in_range():
    a = fm.uniform("t", 3, 1000, "cpu")
    b = fm.uniform("t", 3, 1000, "cpu")
    c = fm.uniform("t", 4, 1000, "cpu")
    assert torch.equal(a, b) and not torch.equal(a, c)
    assert float(a.min()) >= -1.0 and float(a.max()) < 1.0
    assert abs(float(a.mean())) < 0.1 and abs(float(a.std()) - 1 / 3 ** 0.5) < 0.05
    # chunk boundaries do not change values
    n = fm._CHUNK + 5
    big = fm.uniform("t", 3, n, "cpu")
    assert torch.equal(big[:1000], a)
    # values are multiples of 2^-23 and exact in f32: the same bits on any device
    assert torch.equal((a * (1 << 23)).round() / (1 << 23), a)


def test_checksum_is_order_sensitive():
    t = torch.arange(100, dtype=torch.int16)
    assert fm.tensor_checksum(t) == fm.tensor_checksum(t.clone())
    assert fm.tensor_checksum(t) != fm.tensor_checksum(t.flip(0))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_cut_sizes(world):
    # the rank's shard sizes the runtime checks (layer_tensor_bytes in g4_runtime.cu)
    fake = {}
    for full in (False, True):
        q_rows, k_rows, d = (fm.QF, fm.PF, fm.DF) if full else (fm.QS, fm.PS, fm.DS)
        t = {"self_attn.q_proj.weight": torch.zeros(q_rows * fm.H, dtype=torch.uint8),
             "self_attn.q_proj.weight_scale": torch.zeros(q_rows, dtype=torch.bfloat16),
             "self_attn.k_proj.weight": torch.zeros(k_rows * fm.H, dtype=torch.uint8),
             "self_attn.k_proj.weight_scale": torch.zeros(k_rows, dtype=torch.bfloat16),
             "self_attn.o_proj.weight": torch.zeros(fm.H * q_rows, dtype=torch.uint8),
             "mlp.gate_proj.weight_packed": torch.zeros(fm.L * fm.H // 2, dtype=torch.uint8),
             "mlp.up_proj.weight_packed": torch.zeros(fm.L * fm.H // 2, dtype=torch.uint8),
             "mlp.gate_proj.weight_scale": torch.zeros(fm.L * fm.H // 16, dtype=torch.uint8),
             "mlp.up_proj.weight_scale": torch.zeros(fm.L * fm.H // 16, dtype=torch.uint8),
             "mlp.down_proj.weight_packed": torch.zeros(fm.H * fm.L // 2, dtype=torch.uint8),
             "mlp.down_proj.weight_scale": torch.zeros(fm.H * fm.L // 16, dtype=torch.uint8)}
        if not full:
            t["self_attn.v_proj.weight"] = torch.zeros(k_rows * fm.H, dtype=torch.uint8)
            t["self_attn.v_proj.weight_scale"] = torch.zeros(k_rows, dtype=torch.bfloat16)
        s = fm.shard_layer(t, 5 if full else 0, 1, world)
        assert s["self_attn.q_proj.weight"].numel() == q_rows // world * fm.H
        assert s["self_attn.o_proj.weight"].numel() == fm.H * q_rows // world
        assert s["self_attn.k_proj.weight"].numel() == (fm.PF if full else fm.PS // world) * fm.H
        assert s["mlp.down_proj.weight_scale"].numel() == fm.H * fm.L // world // 16
        fake[full] = s
    assert fake[False]["self_attn.v_proj.weight"].numel() == fm.PS // world * fm.H


def test_oracle_rope_tables_follow_rope_data():
    # src/host/runtime.rs:271-299: angle pos / theta^(2i/dim) in f32, identity past the
    # rotated angles; position 0 is cos 1, sin 0 everywhere
    c, s = om.rope_tables(fm.DF, 1_000_000.0, 128, 0)
    assert torch.equal(c, torch.ones(fm.DF)) and torch.equal(s, torch.zeros(fm.DF))
    c, s = om.rope_tables(fm.DF, 1_000_000.0, 128, 777)
    assert torch.equal(c[64:256], torch.ones(192)) and torch.equal(s[64:256], torch.zeros(192))
    assert torch.equal(c[:256], c[256:]) and torch.equal(s[:256], s[256:])
    ang = np.float32(777) / np.power(np.float32(1e6), np.float32(2 * 3) / np.float32(512), dtype=np.float32)
    assert float(c[3]) == float(torch.tensor(np.cos(ang, dtype=np.float32)).to(torch.bfloat16))


def test_oracle_softmax_attention_is_a_weighted_mean():
    q = torch.tensor([[1.0, 0.0], [0.0, 0.0]])
    k = torch.tensor([[1.0, 0.0], [0.0, 1.0]])
    v = torch.tensor([[2.0, 0.0], [0.0, 4.0]])
    out = om.softmax_attend(q, k, v)
    e = np.exp(1.0)
    assert abs(float(out[0, 0]) - 2 * e / (e + 1)) < 1e-2
    assert torch.equal(out[1], torch.tensor([1.0, 2.0]))


def test_golden_fixture_is_consistent():
    path = fm.__file__  # noqa: F841
    from pathlib import Path

    g = np.load(Path(__file__).parent / "golden" / "model_golden.npz")
    for case in ("six_layers_long", "full_depth"):
        spec = g[f"{case}.spec"]
        n_prompt, n_new = int(spec[3]), int(spec[4])
        assert g[f"{case}.prompt"].shape == (n_prompt,)
        assert g[f"{case}.tokens"].shape == (n_new,)
        top = g[f"{case}.top8"]
        assert top.shape == (n_new, 16)
        # the greedy token of each step is the lowest index among the step's maximal logits
        for j, tok in enumerate(g[f"{case}.tokens"].tolist()):
            best = top[j, 0]
            tied = top[j, 8:][top[j, :8] == best].astype(np.int64)
            assert tok == tied.min(), (case, j)
        assert (np.diff(top[:, :8], axis=1) <= 0).all()
        # the small norm-weight tensors regenerate to the recorded checksums
        names = list(g[f"{case}.checksum_names"])
        sums = dict(zip(names, g[f"{case}.checksums"]))
        m_seed = int(spec[2])
        fn = fm._norm_w("final_norm", m_seed, fm.H, "cpu").float()
        fn = (fn * torch.where(fm.uniform("final_norm.sign", m_seed, fm.H, "cpu") < 0, -1.0, 1.0)).to(torch.bfloat16)
        assert fm.tensor_checksum(fn) == int(sums["final_norm"])


# ------------------------------------------------------------------ checkpoint checks
def test_checkpoint_check_accepts_the_reference_layout(tmp_path):
    from g4formats import checkpoint

    p = tmp_path / "ok.safetensors"
    checkpoint.sparse_skeleton(str(p), 6)
    for world in (1, 2, 4, 8):
        assert runtime.check_checkpoint(p, 6, world) == (True, "")
    ok, msg = runtime.check_checkpoint(p, 7, 1)  # a 7th layer is not in the file
    assert not ok and "layers.6." in msg and "missing" in msg


@pytest.mark.parametrize("case", ["missing", "dtype", "shape", "scale_zero", "garbage"])
def test_checkpoint_check_names_the_bad_tensor(tmp_path, case):
    from g4formats import checkpoint

    p = tmp_path / f"{case}.safetensors"
    target = "model.language_model.layers.0.self_attn.q_proj.weight"

    def edit(name, rec):
        if name != target:
            return rec
        if case == "missing":
            return None
        if case == "dtype":
            return dict(rec, dtype="U8")
        if case == "shape":
            return dict(rec, shape=[rec["shape"][1], rec["shape"][0]])
        return rec

    if case == "garbage":
        p.write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{not json at all")
        ok, msg = runtime.check_checkpoint(p, 1)
        assert not ok and "header" in msg
        return
    checkpoint.sparse_skeleton(str(p), 1, global_scale=0.0 if case == "scale_zero" else 9600.0, edit=edit)
    ok, msg = runtime.check_checkpoint(p, 1)
    assert not ok
    if case == "scale_zero":
        assert "invalid NVFP4 global scale" in msg and "weight_global_scale" in msg
    else:
        assert target in msg, msg
    ok, msg = runtime.check_checkpoint(tmp_path / "nope.safetensors", 1)
    assert not ok and "cannot open" in msg
