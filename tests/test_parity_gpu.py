"""Parity of the CUDA path with the reference, through the C ABI, on a B200.

Every text case of the reference's kernel test (src/bin/test_kernels.rs:399-495) runs on
the same byte-identical inputs and is compared with the reference's own expected output
(tests/golden/reference_fixtures.npz, written by scripts/generate_references.py):
  - the reference's pass rule: |got - want| <= atol + 2e-2*|want| per element, with the
    reference's per-case atol (test_kernels.rs:397-495);
  - relative L2 <= 1e-2, and max-abs <= 2e-2 on the MLP block.
"""

import numpy as np
import pytest

from oracle import cases, prng

pytestmark = pytest.mark.gpu

CASES = list(cases.BUILDERS)
REL_L2 = 1e-2


CASE_KERNELS = [(n, "auto") for n in CASES] + [("decoder_feedforward", "stream")]


@pytest.mark.parametrize("name,kernel", CASE_KERNELS)
def test_reference_case(gpu_ctx, golden, name, kernel):
    import harness

    c = harness.build_case(name)
    gpu_ctx.set_mlp_kernel(kernel)  # decoder_feedforward through both kernels ("auto" = tcgen05)
    try:
        got = harness.RUNNERS[name](gpu_ctx, c)
    finally:
        gpu_ctx.set_mlp_kernel("auto")
    if name == "final_norm_and_logits":
        assert got["_lm_checksum"] == int(golden[f"{name}.check.lm_head_weight"][0])
    labels = [k[len(name) + 1:] for k in golden.files if k.startswith(name + ".expected")]
    assert labels
    for label in labels:
        want = prng.bf16_to_f32(golden[f"{name}.{label}"])
        r = cases.compare(want, got[label], cases.ATOL[name])
        print(name, label, r)
        assert r["ok"], (name, label, r)
        assert r["rel_l2"] <= REL_L2, (name, label, r)
        if name == "decoder_feedforward":
            assert r["max_abs"] <= 2e-2, r
    assert gpu_ctx.poll() == 0
