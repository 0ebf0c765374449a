"""Pure-Python XXH64 (fallback when the ``xxhash`` package is missing).

Implements the public XXH64 specification (Yann Collet, xxHash, "XXH64 algorithm
overview": four 64-bit lanes, 32-byte stripes, merge rounds and avalanche).  Used only
as a fallback: the block manager prefers the ``xxhash`` C library, and a unit test
checks the two agree.
"""
from __future__ import annotations

import struct

_M = (1 << 64) - 1
P1 = 0x9E3779B185EBCA87
P2 = 0xC2B2AE3D27D4EB4F
P3 = 0x165667B19E3779F9
P4 = 0x85EBCA77C2B2AE63
P5 = 0x27D4EB2F165667C5


def _rotl(x: int, r: int) -> int:
    return ((x << r) | (x >> (64 - r))) & _M


def _round(acc: int, lane: int) -> int:
    acc = (acc + lane * P2) & _M
    acc = _rotl(acc, 31)
    return (acc * P1) & _M


def _merge(acc: int, val: int) -> int:
    acc ^= _round(0, val)
    return (acc * P1 + P4) & _M


def xxh64_bytes(data: bytes, seed: int = 0) -> int:
    n = len(data)
    p = 0
    if n >= 32:
        v1 = (seed + P1 + P2) & _M
        v2 = (seed + P2) & _M
        v3 = seed & _M
        v4 = (seed - P1) & _M
        limit = n - 32
        while p <= limit:
            a, b, c, d = struct.unpack_from("<4Q", data, p)
            v1 = _round(v1, a)
            v2 = _round(v2, b)
            v3 = _round(v3, c)
            v4 = _round(v4, d)
            p += 32
        h = (_rotl(v1, 1) + _rotl(v2, 7) + _rotl(v3, 12) + _rotl(v4, 18)) & _M
        h = _merge(h, v1)
        h = _merge(h, v2)
        h = _merge(h, v3)
        h = _merge(h, v4)
    else:
        h = (seed + P5) & _M
    h = (h + n) & _M
    while p + 8 <= n:
        (k,) = struct.unpack_from("<Q", data, p)
        h ^= _round(0, k)
        h = (_rotl(h, 27) * P1 + P4) & _M
        p += 8
    if p + 4 <= n:
        (k,) = struct.unpack_from("<I", data, p)
        h ^= (k * P1) & _M
        h = (_rotl(h, 23) * P2 + P3) & _M
        p += 4
    while p < n:
        h ^= (data[p] * P5) & _M
        h = (_rotl(h, 11) * P1) & _M
        p += 1
    h ^= h >> 33
    h = (h * P2) & _M
    h ^= h >> 29
    h = (h * P3) & _M
    h ^= h >> 32
    return h
