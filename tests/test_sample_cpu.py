"""The top-k / top-p sampler's oracle and the device algorithm's building blocks, without
a GPU: the reference's rules (src/host/sampling.rs:20-72) on small cases, the total order
of bf16 logits, the bitonic network of the select/sample kernels restated in numpy, and
the two-level candidate scheme (per-CTA top-kk, then the top-kk of the union)."""

import numpy as np
import pytest

from oracle import prng
from oracle import sampling as smp


def _bits(vals) -> np.ndarray:
    return prng.bf16_bits(np.asarray(vals, dtype=np.float32)).astype(np.uint16)


def test_top1_and_cold_temperature_are_argmax():
    rng = np.random.default_rng(0)
    b = _bits(rng.standard_normal(1000) * 3)
    want = int(smp.ranked_ids(b, 1)[0])
    for u in (0.0, 0.5, 0.999):
        assert smp.sample(b, 1.0, 1, 0.95, [], u) == want
        assert smp.sample(b, 1e-9, 64, 1.0, [], u) == want


def test_equal_logits_rank_by_lower_id_and_zero_signs_follow_total_order():
    b = _bits([1.0, 2.0, 2.0, 2.0, 0.0])
    assert list(smp.ranked_ids(b, 3)) == [1, 2, 3]
    z = np.array([0x8000, 0x0000], dtype=np.uint16)  # -0.0, +0.0
    assert list(smp.ranked_ids(z, 2)) == [1, 0]


def test_banned_ids_are_skipped_unless_all_are_banned():
    b = _bits([5.0, 4.0, 3.0, -1.0])
    assert smp.sample(b, 1e-6, 2, 1.0, [0], 0.0) == 1
    assert smp.sample(b, 1e-6, 1, 1.0, [0, 1], 0.0) == 2
    b2 = _bits([5.0, 4.0])
    assert smp.sample(b2, 1e-6, 1, 1.0, [0, 1], 0.0) == 0  # everything banned: keep all


def test_nucleus_and_draw_follow_the_probabilities():
    b = _bits(np.log(np.array([0.5, 0.3, 0.15, 0.05])))
    # top_p 0.8: nucleus {0, 1}; draws split 0.5 / 0.3 of its 0.8
    picks = [smp.sample(b, 1.0, 4, 0.8, [], u) for u in np.linspace(0, 0.999, 1000)]
    frac0 = picks.count(0) / len(picks)
    assert set(picks) == {0, 1} and abs(frac0 - 0.625) < 0.01


def _bitonic_desc(k: np.ndarray) -> np.ndarray:
    """The kernels' network: for size 2..n, stride size/2..1, pair (lo, lo + stride) with
    lo = 2 i - (i mod stride), descending where lo & size == 0."""
    k = k.copy()
    n = k.size
    size = 2
    while size <= n:
        stride = size >> 1
        while stride > 0:
            i = np.arange(n // 2)
            lo = 2 * i - (i & (stride - 1))
            hi = lo + stride
            desc = (lo & size) == 0
            a, b = k[lo], k[hi]
            swap = (a < b) == desc
            k[lo] = np.where(swap, b, a)
            k[hi] = np.where(swap, a, b)
            stride >>= 1
        size <<= 1
    return k


@pytest.mark.parametrize("n", [2, 64, 2048])
def test_bitonic_network_sorts_descending(n):
    rng = np.random.default_rng(n)
    k = rng.integers(0, 2 ** 62, n, dtype=np.int64)
    np.testing.assert_array_equal(_bitonic_desc(k), np.sort(k)[::-1])


def test_two_level_candidates_equal_the_global_top():
    rng = np.random.default_rng(3)
    b = _bits(np.round(rng.standard_normal(262144) * 4, 1))  # many equal logits
    key = (smp.total_order_key(b) << 32) | (0xFFFFFFFF - np.arange(b.size, dtype=np.int64))
    kk = 66
    cand = np.concatenate([np.sort(key[c:c + 2048])[::-1][:kk] for c in range(0, b.size, 2048)])
    top = np.sort(cand)[::-1][:kk]
    ids = 0xFFFFFFFF - (top & 0xFFFFFFFF)
    np.testing.assert_array_equal(ids, smp.ranked_ids(b, kk))
