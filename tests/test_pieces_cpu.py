"""The activation expansion of the tcgen05 decoder_feedforward kernel, restated in numpy.

`mlp_tc_kernel` (furiosa-opt-gemma4-12b_b200/csrc/g4_mlp_tc.cu, `split_block`) feeds the
bf16 activation to the block-scaled FP4 MMA as 16 e2m1 "pieces".  Each element is aligned
to its 16-element block's exponent eb as a 32-bit fixed-point magnitude T
(|x| = T * 2^(eb - 158)); piece n holds bits (31-2n, 30-2n) of T as the e2m1 values
{0, 0.5, 1, 1.5} with the element's sign, the block scale is 2^(eb - gmax) and the piece's
column scale 2^(gmax - 127 - 2n).  These tests check that the sum over pieces gives back
every element exactly when it is within 2^24 of its block's largest (and within 2^33 of
the vector's), that smaller ones are truncated toward zero by less than 2^-23 of the block
maximum, and that the block scale is always a representable ue4m3 power of two.  The GPU
parity tests check the kernel itself against the oracle."""

import numpy as np

E2M1_VALUE = np.array([0.0, 0.5, 1.0, 1.5])


def bf16_fields(x):
    """Sign, biased exponent and 8-bit significand of bf16-representable f32 values."""
    u = (np.asarray(x, np.float32).view(np.uint32) >> 16).astype(np.int64)
    sign = u >> 15
    e = (u >> 7) & 0xFF
    m = u & 0x7F
    sig = np.where(e > 0, m | 0x80, m)
    ex = np.where(e > 0, e, 1)
    return sign, ex, sig


def split_vector(x):
    """Pieces of a vector (length a multiple of 16): codes [n, K], block exponents and gmax."""
    x = np.asarray(x, np.float32)
    sign, ex, sig = bf16_fields(x)
    gmax = int(((np.float32(np.abs(x).max()) * np.float32(1.01)).view(np.uint32) >> 23) & 0xFF)
    blocks = x.size // 16
    ex_b = ex.reshape(blocks, 16)
    sig_b = sig.reshape(blocks, 16)
    eb = np.where(sig_b > 0, ex_b, 0).max(axis=1)
    eb = np.maximum(eb, gmax - 9)
    off = eb[:, None] - ex_b
    t = np.where(
        (sig_b == 0) | (off >= 32),
        0,
        np.where(off <= 24, sig_b << np.clip(24 - off, 0, 31), sig_b >> np.clip(off - 24, 0, 63)),
    ).astype(np.int64)
    assert (t < 2**32).all()
    codes = np.stack([(t >> (30 - 2 * n)) & 3 for n in range(16)])  # [16, blocks, 16]
    return codes.reshape(16, -1), sign, eb, gmax


def rebuild(codes, sign, eb, gmax):
    """Sum over pieces of value * block scale * column scale, in exact float64."""
    blocks = eb.size
    block_scale = np.repeat(np.exp2((eb - gmax).astype(np.float64)), 16)
    total = np.zeros(blocks * 16)
    for n in range(16):
        total += E2M1_VALUE[codes[n]] * block_scale * np.exp2(gmax - 127 - 2 * n)
    return np.where(sign == 1, -total, total)


def ue4m3_pow2_ok(k):
    return -9 <= k <= 0  # 2^-9 .. 2^0: subnormal ue4m3 below 2^-6, normal above


def bf16_round(x):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return u.astype(np.uint32).view(np.float32)


def check(x):
    codes, sign, eb, gmax = split_vector(x)
    assert all(ue4m3_pow2_ok(int(k)) for k in eb - gmax)
    y = rebuild(codes, sign, eb, gmax)
    x64 = x.astype(np.float64)
    blk_max = np.repeat(np.abs(x64).reshape(-1, 16).max(axis=1), 16)
    vec_max = np.abs(x64).max()
    near = (np.abs(x64) >= blk_max * 2.0**-24) & (np.abs(x64) >= vec_max * 2.0**-33)
    assert np.array_equal(y[near], x64[near])
    err = x64 - y
    assert (np.sign(err[~near]) * np.sign(x64[~near]) >= 0).all()  # truncation toward zero
    assert (np.abs(err) <= np.maximum(blk_max, vec_max * 2.0**-9) * 2.0**-23).all()
    return y


def test_pieces_rebuild_normal_activations_exactly():
    rng = np.random.default_rng(0)
    for scale in (1e-3, 1.0, 37.0, 3e4):
        x = bf16_round(rng.standard_normal(15360).astype(np.float32) * scale)
        y = check(x)
        assert np.array_equal(y, x.astype(np.float64))


def test_pieces_wide_range_zeros_and_subnormals():
    rng = np.random.default_rng(1)
    octaves = rng.integers(-30, 8, size=3840)
    x = rng.standard_normal(3840) * np.exp2(octaves)
    x[::7] = 0.0
    x[5] = -0.0
    x[100:116] = 0.0  # an all-zero block
    x[200] = 2.0**-130  # bf16 subnormal
    check(bf16_round(x.astype(np.float32)))


def test_pieces_block_scale_clamp():
    # a block far below the vector's largest element takes the clamped exponent gmax - 9
    x = np.zeros(64, np.float32)
    x[0] = 1000.0
    x[16:32] = bf16_round(np.linspace(-1e-3, 1e-3, 16).astype(np.float32))
    x[32:48] = 2.0**-40
    check(bf16_round(x))
