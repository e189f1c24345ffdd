"""The stream-K work split of the tcgen05 decoder_feedforward kernel, restated in Python.

`mlp_tc_kernel` (furiosa-opt-gemma4-12b_b200/csrc/g4_mlp_tc.cu, struct Part) cuts each
phase's (tile, 256-k stage) pairs into one contiguous range per CTA, the last CTA's
range 1/8 shorter in the gate/up phase (d = 1: it starts last, on the SM the previous
launch's tail occupied).  The kernel holds at most kMaxCtaSeg segments (runs inside one
tile) per CTA and phase, kMaxSeg segments per tile, and kMaxLocal resident k-stages of
activation pieces; the launcher checks these on the host and refuses a split that breaks
them.  These tests check that the shapes the library runs (one GPU on 148 SMs, and the
tensor-parallel shards TP2 / TP4) fit, that the ranges tile the work exactly once, and
that every index the kernel derives stays inside its buffers."""

import pytest

H, L = 3840, 15360
K_STAGE, MAX_CTA_SEG, MAX_SEG, MAX_LOCAL = 256, 4, 8, 16
TC_TILES = L // 64 + H // 128          # kTcTiles
PART_WORDS = TC_TILES * MAX_SEG * 128   # kTcPartWords (tagged partials of both phases)
SEG_FLOATS = H                          # kTcSegFloats: the down projection's H sums


class Part:
    def __init__(self, T, S, d):
        self.T, self.S, self.W, self.d = T, S, T * S, d

    def lo(self, c, G):
        return self.W if c >= G else (c * 8 * self.W) // (8 * G - self.d)

    def owner(self, i, G):
        c = ((i + 1) * (8 * G - self.d) - 1) // (8 * self.W)
        return min(c, G - 1)


def phases(lrows):
    return [Part(lrows // 64, H // K_STAGE, 1), Part(H // 128, lrows // K_STAGE, 0)]


@pytest.mark.parametrize("tp", [1, 2, 4])
@pytest.mark.parametrize("G", [148, 132])
def test_partition_fits_the_kernel(tp, G):
    lrows = L // tp
    for ph, P in enumerate(phases(lrows)):
        covered = []
        for c in range(G):
            lo, hi = P.lo(c, G), P.lo(c + 1, G)
            n = hi - lo
            assert n >= 1, (ph, c)
            assert not (P.S > MAX_LOCAL and n > MAX_LOCAL), (ph, c, n)   # resident window
            assert n // P.S + 2 <= MAX_CTA_SEG, (ph, c, n)                # segments per CTA
            covered.extend(range(lo, hi))
            # owner() agrees with the ranges
            assert P.owner(lo, G) == c and P.owner(hi - 1, G) == c
        assert covered == list(range(P.W))                                # every pair once
        for t in range(P.T):
            nseg = P.owner(t * P.S + P.S - 1, G) - P.owner(t * P.S, G) + 1
            assert 1 <= nseg <= MAX_SEG, (ph, t, nseg)


def test_last_cta_gets_a_lighter_gate_up_share():
    G = 148
    P0 = phases(L)[0]
    sizes = [P0.lo(c + 1, G) - P0.lo(c, G) for c in range(G)]
    assert sizes[-1] < min(sizes[:-1])
    assert sizes[-1] >= 0.8 * (P0.W / G)


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_buffer_indices_stay_in_bounds(tp):
    lrows = L // tp
    P0, P1 = phases(lrows)
    # tagged partials: ((phase-1 tiles after the gate/up ones) tile * kMaxSeg + segment) * 128 + row
    assert (P0.T + P1.T - 1) * MAX_SEG * 128 + (MAX_SEG - 1) * 128 + 127 < PART_WORDS
    # tagged h: tile * 64 + row of a gate/up tile; read back per 256-k stage of the down phase
    assert (P0.T - 1) * 64 + 63 < L and P1.S * K_STAGE <= L
    # the down projection's sums: tile * 128 + row of a down tile
    assert (P1.T - 1) * 128 + 127 < H <= SEG_FLOATS
    # TMA: 16-byte rows of the down projection's scales, 128-byte boxes of its codes
    assert (lrows // 16) % 16 == 0 and (lrows // 2) % 128 == 0
    # the whole down phase is staged at once when it fits the resident pieces
    if P1.S <= MAX_LOCAL:
        assert P1.S * 16 <= 320  # one block of 16 per staging thread


def test_tp8_shard_does_not_fit_a_tensor_map():
    lrows = L // 8
    assert (lrows // 16) % 16 != 0  # 120-byte scale rows: the streaming kernel serves TP8
