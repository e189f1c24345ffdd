"""Stateless tensor synthesis -- a numpy restatement of the reference's `fixture_prng`.

TEST INFRASTRUCTURE ONLY: imported by tests/, `__graft_entry__.smoke()` and bench.py's
CPU-baseline leg to build inputs and check results.  The product path never uses it.

Every input of every kernel case is synthesized from the tensor's *name* and each
element's *index*, byte-identically to the reference (scripts/fixture_prng.py and the
`prng` module of src/bin/test_kernels.rs:10-124), so no input ever needs storing:
  word(name, i) = splitmix64-style mix of (FNV-1a(name) ^ i)    fixture_prng.py:46-69
  u01(w)        = top 24 bits / 2^24 (exact in f32)             fixture_prng.py:73-79
  bf16 rounding = explicit round-half-to-even on the f32 bits   fixture_prng.py:82-92
  f8 codes      = sign | exponent band | mantissa bit fields    fixture_prng.py:130-150
  f4 codes      = top nibble of each element's word, packed     fixture_prng.py:153-168
  checksum      = sum of u32 words * (2*index + 1) mod 2^32     fixture_prng.py:172-200
The constants of the hash are the reference's (they define the byte stream); the code
here is organised around a single `_mix` of a uint64 index array.
"""

from __future__ import annotations

import numpy as np

_U64 = np.uint64
_FNV_BASIS = 0xCBF29CE484222325
_FNV_MULT = 0x100000001B3
_INC = _U64(0x9E3779B97F4A7C15)
_M1 = _U64(0xBF58476D1CE4E5B9)
_M2 = _U64(0x94D049BB133111EB)
_WORD_BLOCK = 1 << 23


def name_seed(name: str) -> int:
    """FNV-1a over the UTF-8 name (fixture_prng.py:46-56), as a Python int."""
    h = _FNV_BASIS
    for b in name.encode("utf-8"):
        h = ((h ^ b) * _FNV_MULT) & 0xFFFFFFFFFFFFFFFF
    return h


def _mix(seed: int, first: int, count: int) -> np.ndarray:
    """Words `first .. first+count-1` of the stream `seed` (fixture_prng.py:59-69)."""
    z = (np.arange(first, first + count, dtype=_U64) ^ _U64(seed)) + _INC
    z = (z ^ (z >> _U64(30))) * _M1
    z = (z ^ (z >> _U64(27))) * _M2
    return z ^ (z >> _U64(31))


def words(name: str, count: int, offset: int = 0) -> np.ndarray:
    return _mix(name_seed(name), offset, count)


def unit_f32(w: np.ndarray) -> np.ndarray:
    """[0,1) with 24 random bits -- k/2^24 is exact in f32 (fixture_prng.py:73-79)."""
    return (w >> _U64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)


def bf16_bits(values: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns, round half to even (fixture_prng.py:82-92).  Finite inputs."""
    u = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32)
    return ((u + (np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1)))) >> np.uint32(16)).astype(
        np.uint16
    )


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_bf16(values: np.ndarray) -> np.ndarray:
    """bf16(x) as f32, round half to even (NaN/Inf passed through as in torch)."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = bf16_to_f32(bf16_bits(v))
    bad = ~np.isfinite(v)
    if bad.any():
        out = out.copy()
        out[bad] = v[bad]
    return out


def bf16_uniform(name: str, count: int, lo: float, hi: float, offset: int = 0) -> np.ndarray:
    """bf16 bits of lo + (hi-lo)*u in f32: one multiply, then one add (fixture_prng.py:96-104)."""
    u = unit_f32(words(name, count, offset))
    lo32, hi32 = np.float32(lo), np.float32(hi)
    span = np.float32(hi32 - lo32)
    return bf16_bits(lo32 + span * u)


def f32_uniform(name: str, count: int, lo: float, hi: float, offset: int = 0) -> np.ndarray:
    u = unit_f32(words(name, count, offset))
    lo32, hi32 = np.float32(lo), np.float32(hi)
    return lo32 + np.float32(hi32 - lo32) * u


def bf16_signs(name: str, count: int, scale: float = 1.0, offset: int = 0) -> np.ndarray:
    """bf16 +/-|scale|, sign = top bit of the word (fixture_prng.py:117-127)."""
    mag = bf16_bits(np.array([abs(scale)], dtype=np.float32))[0]
    neg = (words(name, count, offset) >> _U64(63)).astype(np.uint16)
    return (mag | (neg << np.uint16(15))).astype(np.uint16)


def f8_banded(name: str, count: int, exp_min: int, exp_max: int, signed: bool = True,
              offset: int = 0) -> np.ndarray:
    """E4M3 bytes with exponent in [exp_min, exp_max] (fixture_prng.py:130-150)."""
    if not (0 <= exp_min <= exp_max <= 14):
        raise ValueError(f"{name}: exponent band {exp_min}..{exp_max} out of range")
    w = words(name, count, offset)
    expo = np.uint64(exp_min) + (w >> _U64(32)) % np.uint64(exp_max - exp_min + 1)
    mant = (w >> _U64(56)) & _U64(7)
    out = (expo << _U64(3)) | mant
    if signed:
        out |= (w >> _U64(63)) << _U64(7)
    return out.astype(np.uint8)


def f4_nibbles(name: str, count: int, offset: int = 0) -> np.ndarray:
    """Packed E2M1 codes, two per byte, low nibble = even element (fixture_prng.py:153-168)."""
    if count % 2 or offset % 2:
        raise ValueError(f"{name}: f4 count/offset must be even")
    nib = ((words(name, count, offset) >> _U64(60)) & _U64(0xF)).astype(np.uint8)
    return (nib[0::2] | (nib[1::2] << np.uint8(4))).astype(np.uint8)


def checksum(storage: np.ndarray, word_offset: int = 0) -> int:
    """Position-weighted u32 checksum of the storage bytes (fixture_prng.py:172-200)."""
    raw = np.ascontiguousarray(storage).reshape(-1).view(np.uint8)
    pad = (-raw.size) % 4
    if pad:
        if word_offset:
            raise ValueError("only the final block of a chunked tensor may need padding")
        raw = np.concatenate([raw, np.zeros(pad, dtype=np.uint8)])
    w32 = raw.view(np.uint32)
    total = 0
    for start in range(0, w32.size, _WORD_BLOCK):
        blk = w32[start:start + _WORD_BLOCK]
        idx = np.arange(blk.size, dtype=np.uint32) + np.uint32((word_offset + start) & 0xFFFFFFFF)
        total += int((blk * (idx * np.uint32(2) + np.uint32(1))).sum(dtype=np.uint32))
    return total & 0xFFFFFFFF


# ---------------------------------------------------------------------------- decoding
E2M1_MAGNITUDE = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def e2m1_unpack(packed: np.ndarray) -> np.ndarray:
    """[N, K/2] packed codes -> [N, K] float32 values (generate_references.py:207-216)."""
    p = np.asarray(packed, dtype=np.uint8)
    codes = np.stack([p & 0x0F, p >> 4], axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)
    vals = E2M1_MAGNITUDE[codes & 7]
    return np.where(codes >= 8, -vals, vals).astype(np.float32)


def _e4m3_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 7
        if e == 15 and m == 7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_VALUE = _e4m3_table()


def e4m3_decode(codes: np.ndarray) -> np.ndarray:
    return E4M3_VALUE[np.asarray(codes, dtype=np.uint8)]
