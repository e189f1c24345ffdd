"""CPU oracle of top-k / top-p sampling (src/host/sampling.rs:20-72).

TEST INFRASTRUCTURE ONLY: the checker of g4_sample_top_k_top_p.

Restates `sample` step by step in float32 numpy:
  temperature = max(T, 1e-5); keep = min(top_k + |banned|, n); the `keep` largest logits
  in descending order (Rust's f32::total_cmp: -0.0 below +0.0, NaN by sign); banned ids
  dropped unless that drops all; truncated to top_k; p_i = exp((l_i - l_0) / T) summed
  and divided in order; nucleus = the first prefix whose running sum reaches top_p;
  threshold = u * (sum of the nucleus); the first id whose running sum reaches it, else
  the nucleus's last.
The reference's `select_nth_unstable_by` / `sort_unstable_by` leave the order of equal
logits open; here (and in the library) equal logits rank by lower id.
"""

from __future__ import annotations

import numpy as np

f32 = np.float32


def total_order_key(bits: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> integers ordered like f32::total_cmp of their values."""
    b = np.asarray(bits, dtype=np.uint32) & 0xFFFF
    return np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000).astype(np.int64)


def ranked_ids(bits: np.ndarray, keep: int) -> np.ndarray:
    """The `keep` ids of largest logit, descending; equal logits by lower id."""
    key = total_order_key(bits)
    order = np.lexsort((np.arange(key.size), -key))
    return order[:keep]


def sample(bits: np.ndarray, temperature: float, top_k: int, top_p: float, banned, u: float) -> int:
    """bits: bf16 bit patterns of the logits [n] (uint16)."""
    bits = np.asarray(bits, dtype=np.uint16)
    n = bits.size
    logits = (bits.astype(np.uint32) << 16).view(np.float32)
    t = f32(max(temperature, 1e-5))
    banned = list(banned)
    keep = min(top_k + len(banned), n)
    ranked = [int(i) for i in ranked_ids(bits, keep)]
    if banned:
        filtered = [i for i in ranked if i not in set(banned)]
        if filtered:
            ranked = filtered
    ranked = ranked[:min(top_k, len(ranked))]
    mx = logits[ranked[0]]
    probs = [f32(np.exp(f32(f32(logits[i] - mx) / t))) for i in ranked]
    total = f32(0.0)
    for p in probs:
        total = f32(total + p)
    probs = [f32(p / total) for p in probs]
    nucleus = len(probs)
    cum = f32(0.0)
    for i, p in enumerate(probs):
        cum = f32(cum + p)
        if cum >= f32(top_p):
            nucleus = i + 1
            break
    nsum = f32(0.0)
    for p in probs[:nucleus]:
        nsum = f32(nsum + p)
    threshold = f32(f32(u) * nsum)
    acc = f32(0.0)
    for i, p in enumerate(probs[:nucleus]):
        acc = f32(acc + p)
        if acc >= threshold:
            return ranked[i]
    return ranked[nucleus - 1]


def boundary_gap(bits: np.ndarray, temperature: float, top_k: int, top_p: float, banned, u: float) -> float:
    """How close the draw's threshold lies to a running-sum boundary of the nucleus
    (relative): where exp's last-bit differences between two libraries can move a pick."""
    bits = np.asarray(bits, dtype=np.uint16)
    logits = (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    keep = min(top_k + len(banned), bits.size)
    ranked = [int(i) for i in ranked_ids(bits, keep) if int(i) not in set(banned)][:top_k]
    p = np.exp((logits[ranked] - logits[ranked[0]]) / max(temperature, 1e-5))
    p /= p.sum()
    c = np.cumsum(p)
    nucleus = int(np.searchsorted(c, top_p - 1e-7) + 1)
    c = c[:nucleus] / c[nucleus - 1]
    return float(np.min(np.abs(c - u)))


def runtime_draw(seed: int, pos: int) -> float:
    """The decode runtime's draw for the step at `pos` (g4_workspace_set_sampling):
    splitmix64 of seed + pos * 0x9E3779B97F4A7C15, top 24 bits / 2^24."""
    m = (1 << 64) - 1
    z = (seed + (pos & 0xFFFFFFFF) * 0x9E3779B97F4A7C15) & m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    z ^= z >> 31
    return float(np.float32(z >> 40) * np.float32(1.0 / 16777216.0))
