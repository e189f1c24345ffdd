#!/usr/bin/env python3
"""Regenerate `tests/golden/reference_fixtures.npz` from the reference's own generator.

This script imports the reference project's `scripts/generate_references.py` (the torch
file that writes the reference's `ref/fixtures.safetensors`) and runs its text-decoder
generators unchanged.  It needs the reference checkout, so it only runs where that is
mounted; the GPU box and the test suite read the committed `.npz`, never the reference.

One adapter is needed.  The generator imports `transformers.models.gemma4_unified`
(generate_references.py:56-69); the installed transformers 5.5 ships the same text
modules under `transformers.models.gemma4` (`Gemma4RMSNorm` with `with_scale`,
`Gemma4TextMLP`, `Gemma4TextRotaryEmbedding` with "proportional" RoPE,
`Gemma4TextScaledWordEmbedding`, `apply_rotary_pos_emb`).  The adapter registers a
`gemma4_unified` alias module that maps each `Gemma4Unified*` name to the `Gemma4*`
class.  The vision/audio classes are stubs because the vision/audio generators are
not run (they are outside the text hot path).  `verify_rope_matches_upstream`
(generate_references.py:273-290) still runs and guards the RoPE table convention.

Usage:  python tests/golden/make_golden.py <reference checkout>   (or G4B200_REFERENCE_DIR=...)
"""

import sys
import time
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_fixtures.npz"

# The text generators of generate_references.py:762-782 that cover the hot path.
TEXT_TESTS = [
    "embed_token",
    "copy_hidden_state",
    "sliding_project_qkv_exact",
    "sliding_project_qkv_random",
    "sliding_attention",
    "sliding_attention_output_exact",
    "sliding_attention_output_random",
    "full_project_qkv_exact",
    "full_project_qkv_random",
    "full_attention",
    "full_attention_output_exact",
    "full_attention_output_random",
    "decoder_feedforward",
    "final_norm_and_logits",
]


def install_gemma4_unified_alias() -> None:
    """Register `transformers.models.gemma4_unified` as an alias of `gemma4`."""
    from transformers.models.gemma4 import configuration_gemma4 as cfg
    from transformers.models.gemma4 import modeling_gemma4 as mdl

    class _Unavailable:
        def __init__(self, *args, **kwargs):
            raise RuntimeError("vision/audio modules are not part of the text hot path")

    pkg = types.ModuleType("transformers.models.gemma4_unified")
    conf = types.ModuleType("transformers.models.gemma4_unified.configuration_gemma4_unified")
    model = types.ModuleType("transformers.models.gemma4_unified.modeling_gemma4_unified")
    conf.Gemma4UnifiedTextConfig = cfg.Gemma4TextConfig
    conf.Gemma4UnifiedAudioConfig = _Unavailable
    conf.Gemma4UnifiedVisionConfig = _Unavailable
    model.Gemma4UnifiedRMSNorm = mdl.Gemma4RMSNorm
    model.Gemma4UnifiedTextMLP = mdl.Gemma4TextMLP
    model.Gemma4UnifiedTextRotaryEmbedding = mdl.Gemma4TextRotaryEmbedding
    model.Gemma4UnifiedTextScaledWordEmbedding = mdl.Gemma4TextScaledWordEmbedding
    model.apply_rotary_pos_emb = mdl.apply_rotary_pos_emb
    model.Gemma4UnifiedMultimodalEmbedder = _Unavailable
    model.Gemma4UnifiedVisionEmbedder = _Unavailable
    pkg.configuration_gemma4_unified = conf
    pkg.modeling_gemma4_unified = model
    sys.modules[pkg.__name__] = pkg
    sys.modules[conf.__name__] = conf
    sys.modules[model.__name__] = model


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    """Exact bf16 bit patterns of a tensor whose values are all bf16-representable."""
    b = t.detach().to(torch.bfloat16)
    if not torch.equal(b.float(), t.detach().float()):
        raise AssertionError("expected output is not bf16-valued")
    return b.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def main() -> None:
    import os

    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("G4B200_REFERENCE_DIR")
    if not ref:
        raise SystemExit("usage: make_golden.py <reference checkout> (or set G4B200_REFERENCE_DIR)")
    reference = Path(ref)
    scripts = reference / "scripts"
    if not (scripts / "generate_references.py").exists():
        raise SystemExit(f"reference generator not found under {scripts}")
    install_gemma4_unified_alias()
    sys.path.insert(0, str(scripts))
    import generate_references as gen  # noqa: E402  (the reference's own file)

    torch.set_grad_enabled(False)
    gen.verify_rope_matches_upstream(gen.text_config())
    entries: dict[str, np.ndarray] = {}
    for name in TEXT_TESTS:
        t0 = time.time()
        outputs, checks = gen.TESTS[name]()
        for label, tensor in outputs.items():
            entries[f"{name}.{label}"] = bf16_bits(tensor)
        for label, value in checks.items():
            entries[f"{name}.check.{label}"] = np.array([value], dtype=np.uint32)
        print(f"  {name:34} {', '.join(outputs)}  ({len(checks)} inputs, {time.time() - t0:.1f}s)")
    np.savez_compressed(OUT, **entries)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB, {len(TEXT_TESTS)} tests)")


if __name__ == "__main__":
    main()
