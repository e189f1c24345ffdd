"""g4_sample_top_k_top_p on a B200 against the CPU restatement of the reference's
sampler (oracle/sampling.py, src/host/sampling.rs:20-72).

Full-vocabulary logits (262144, bf16) with many exactly equal values, the Gemma settings
(T 1.0, top_k 64, top_p 0.95, the two suppressed tokens banned) and others; for each, a
spread of uniform draws.  The picked id must be the oracle's; the only tolerated
difference is a draw whose threshold lies within 1e-5 (relative) of a running-sum
boundary, where the device's and numpy's exp may differ in the last bit.
"""

import numpy as np
import pytest
import torch

import g4b200 as g4
from oracle import prng
from oracle import sampling as smp

pytestmark = pytest.mark.gpu

W = 262144
SUPPRESSED = [258880, 258883]  # two ids in the vocabulary, as the reference bans EOI/EOA


def _logits(seed: int, scale: float, quantum: float = 0.0) -> np.ndarray:
    x = np.random.default_rng(seed).standard_normal(W).astype(np.float32) * scale
    if quantum:
        x = np.round(x / quantum) * quantum
    x = np.tanh(x / 30.0) * 30.0  # the softcap's range
    return prng.bf16_bits(x.astype(np.float32)).astype(np.uint16)


CASES = [
    (0, 3.0, 0.0, 1.0, 64, 0.95, SUPPRESSED),
    (1, 3.0, 0.25, 1.0, 64, 0.95, SUPPRESSED),   # many equal logits
    (2, 1.0, 0.0, 0.7, 40, 0.9, []),
    (3, 5.0, 0.0, 1.5, 126, 1.0, SUPPRESSED),
    (4, 3.0, 0.0, 1.0, 1, 0.95, []),
    (5, 0.5, 0.0, 2.0, 16, 0.3, [7, 11, 13]),
]


@pytest.mark.parametrize("case", CASES)
def test_sample_matches_oracle(gpu_ctx, case):
    seed, scale, quantum, temp, top_k, top_p, banned = case
    bits = _logits(seed, scale, quantum)
    if banned:  # make the banned ids the largest logits, so banning matters
        bits[banned] = prng.bf16_bits(np.array([29.5] * len(banned), dtype=np.float32)).astype(np.uint16)
    logits = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    u_dev = torch.zeros(1, dtype=torch.float32, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    same = near = 0
    for u in np.linspace(0.0, 0.995, 24).astype(np.float32):
        u_dev.fill_(float(u))
        g4.sample_top_k_top_p(gpu_ctx, logits, temp, top_k, top_p, banned, u_dev, out)
        torch.cuda.synchronize()
        got = int(out.item())
        want = smp.sample(bits, temp, top_k, top_p, banned, float(u))
        if got == want:
            same += 1
        else:
            gap = smp.boundary_gap(bits, temp, top_k, top_p, banned, float(u))
            assert gap < 1e-5, (case, float(u), got, want, gap)
            near += 1
        assert got not in banned or all(i in banned for i in smp.ranked_ids(bits, top_k + len(banned)))
    print(f"case {seed}: {same} identical, {near} at a boundary")
    assert gpu_ctx.poll() == 0


def test_sample_small_vocab_and_argument_errors(gpu_ctx):
    bits = prng.bf16_bits(np.array([0.5, 3.0, 3.0, -2.0, 1.0], dtype=np.float32)).astype(np.uint16)
    logits = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    u = torch.zeros(1, dtype=torch.float32, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    g4.sample_top_k_top_p(gpu_ctx, logits, 1.0, 100, 1.0, [], u, out)  # top_k beyond n
    torch.cuda.synchronize()
    assert int(out.item()) == 1  # u = 0: the largest logit, lower id of the tie
    for bad in ((1.0, 0, 0.9, []), (1.0, 127, 0.9, [1, 2]), (1.0, 8, 0.0, []), (1.0, 8, 1.5, [])):
        with pytest.raises(g4.G4Error):
            g4.sample_top_k_top_p(gpu_ctx, logits, bad[0], bad[1], bad[2], bad[3], u, out)
    assert gpu_ctx.poll() == 0
