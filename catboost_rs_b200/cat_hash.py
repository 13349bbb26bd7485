"""Category hashes as upstream CatBoost stores them in a model file.

A one-hot feature's model entry lists its categories by CalcCatFeatureHash:
the low 32 bits of CityHash64 (version 1.0) of the category's text
(the reference's crates/cb-data/src/cat_hash.rs).  CityHash64 is restated
here from Google's published CityHash 1.0 description (little-endian 64-bit
reads, the length-class mixers for 0-16, 17-32 and 33-64 bytes, and the
64-byte main loop over two 128-bit states), in Python: a model holds few
categories, so speed does not matter.
"""
from __future__ import annotations

_M = (1 << 64) - 1
_K0 = 0xC3A5C85C97CB3127
_K1 = 0xB492B66FBE98F273
_K2 = 0x9AE16A3B2F90404F
_K3 = 0xC949D7C7509E6557
_KMUL = 0x9DDFEA08EB382D69


def _f64(s: bytes, i: int) -> int:
    return int.from_bytes(s[i:i + 8], "little")


def _f32(s: bytes, i: int) -> int:
    return int.from_bytes(s[i:i + 4], "little")


def _rot(v: int, r: int) -> int:
    return v if r == 0 else ((v >> r) | (v << (64 - r))) & _M


def _rot1(v: int, r: int) -> int:  # r >= 1
    return ((v >> r) | (v << (64 - r))) & _M


def _shift_mix(v: int) -> int:
    return v ^ (v >> 47)


def _hash16(u: int, v: int) -> int:
    a = ((u ^ v) * _KMUL) & _M
    a ^= a >> 47
    b = ((v ^ a) * _KMUL) & _M
    b ^= b >> 47
    return (b * _KMUL) & _M


def _len0to16(s: bytes) -> int:
    n = len(s)
    if n > 8:
        a, b = _f64(s, 0), _f64(s, n - 8)
        return _hash16(a, _rot1((b + n) & _M, n)) ^ b
    if n >= 4:
        a = _f32(s, 0)
        return _hash16((n + (a << 3)) & _M, _f32(s, n - 4))
    if n > 0:
        a, b, c = s[0], s[n >> 1], s[n - 1]
        y = (a + (b << 8)) & 0xFFFFFFFF
        z = (n + (c << 2)) & 0xFFFFFFFF
        return (_shift_mix(((y * _K2) ^ (z * _K3)) & _M) * _K2) & _M
    return _K2


def _len17to32(s: bytes) -> int:
    n = len(s)
    a = (_f64(s, 0) * _K1) & _M
    b = _f64(s, 8)
    c = (_f64(s, n - 8) * _K2) & _M
    d = (_f64(s, n - 16) * _K0) & _M
    return _hash16((_rot((a - b) & _M, 43) + _rot(c, 30) + d) & _M,
                   (a + _rot(b ^ _K3, 20) - c + n) & _M)


def _weak32(w: int, x: int, y: int, z: int, a: int, b: int):
    a = (a + w) & _M
    b = _rot((b + a + z) & _M, 21)
    c = a
    a = (a + x + y) & _M
    b = (b + _rot(a, 44)) & _M
    return (a + z) & _M, (b + c) & _M


def _weak32s(s: bytes, i: int, a: int, b: int):
    return _weak32(_f64(s, i), _f64(s, i + 8), _f64(s, i + 16), _f64(s, i + 24), a, b)


def _len33to64(s: bytes) -> int:
    n = len(s)
    z = _f64(s, 24)
    a = (_f64(s, 0) + (n + _f64(s, n - 16)) * _K0) & _M
    b = _rot((a + z) & _M, 52)
    c = _rot(a, 37)
    a = (a + _f64(s, 8)) & _M
    c = (c + _rot(a, 7)) & _M
    a = (a + _f64(s, 16)) & _M
    vf = (a + z) & _M
    vs = (b + _rot(a, 31) + c) & _M
    a = (_f64(s, 16) + _f64(s, n - 32)) & _M
    z = _f64(s, n - 8)
    b = _rot((a + z) & _M, 52)
    c = _rot(a, 37)
    a = (a + _f64(s, n - 24)) & _M
    c = (c + _rot(a, 7)) & _M
    a = (a + _f64(s, n - 16)) & _M
    wf = (a + z) & _M
    ws = (b + _rot(a, 31) + c) & _M
    r = _shift_mix(((vf + ws) * _K2 + (wf + vs) * _K0) & _M)
    return (_shift_mix((r * _K0 + vs) & _M) * _K2) & _M


def city_hash64(data: bytes) -> int:
    """CityHash64 (version 1.0) of a byte string."""
    s = bytes(data)
    n = len(s)
    if n <= 16:
        return _len0to16(s)
    if n <= 32:
        return _len17to32(s)
    if n <= 64:
        return _len33to64(s)
    x = _f64(s, n - 40)
    y = (_f64(s, n - 16) + _f64(s, n - 56)) & _M
    z = _hash16((_f64(s, n - 48) + n) & _M, _f64(s, n - 24))
    v = _weak32s(s, n - 64, n, z)
    w = _weak32s(s, n - 32, (y + _K1) & _M, x)
    x = (x * _K1 + _f64(s, 0)) & _M
    left = (n - 1) & ~63
    i = 0
    while True:
        x = (_rot((x + y + v[0] + _f64(s, i + 8)) & _M, 37) * _K1) & _M
        y = (_rot((y + v[1] + _f64(s, i + 48)) & _M, 42) * _K1) & _M
        x ^= w[1]
        y = (y + v[0] + _f64(s, i + 40)) & _M
        z = (_rot((z + w[0]) & _M, 33) * _K1) & _M
        v = _weak32s(s, i, (v[1] * _K1) & _M, (x + w[0]) & _M)
        w = _weak32s(s, i + 32, (z + w[1]) & _M, (y + _f64(s, i + 16)) & _M)
        z, x = x, z
        i += 64
        left -= 64
        if left == 0:
            break
    return _hash16((_hash16(v[0], w[0]) + _shift_mix(y) * _K1 + z) & _M, (_hash16(v[1], w[1]) + x) & _M)


def cat_feature_hash(value) -> int:
    """CalcCatFeatureHash of a category: the low 32 bits of CityHash64 of its
    text (str() for non-string values), as an unsigned 32-bit integer."""
    text = value if isinstance(value, str) else str(value)
    return city_hash64(text.encode("utf-8")) & 0xFFFFFFFF
