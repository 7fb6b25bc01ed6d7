"""Threefry2x32-20 counter PRNG and the distributions Sheaf builds on it.

Restates sheaf/src/core/prng.rs (VERSION "threefry2x32-20/16bit-v1") and the
way random ops consume it in sheaf/src/lowering/stablehlo/random_ops.rs:
  * a key is 4 f32 limbs holding 16-bit halves of two u32 words
    (encode/decode, prng.rs:29-55);
  * `random-key s`    -> encode(seed(s))            (random_ops.rs:86-91)
  * `random-split k n` -> child i = threefry(k, [i, 1])  (prng.rs:81-84, random_ops.rs:146-162)
  * sampling bits for flat element index i = threefry(k, [i, 0]) (prng.rs:86-89, random_ops.rs:99-110)
  * uniform = (bits >> 8) * 2^-24                   (prng.rs:91-97)
  * normal  = sqrt(-2 log max(u1, 2^-24)) * cos(2 pi u2)   (prng.rs:99-113)
  * randint = clamp(floor(u * (high-low)) + low, low, high-1)  (prng.rs:115-126)
All float arithmetic is float32, as in the reference.
"""
from __future__ import annotations

import numpy as np

U32 = np.uint32
F32 = np.float32
ROTATIONS = (13, 15, 26, 6, 17, 29, 16, 24)  # prng.rs:66


def seed(s: int) -> tuple[int, int]:
    """prng.rs:27: [seed as u32, (seed as u64 >> 32) as u32]."""
    u = s & 0xFFFFFFFFFFFFFFFF
    return (u & 0xFFFFFFFF, (u >> 32) & 0xFFFFFFFF)


def encode(words) -> np.ndarray:
    """prng.rs:29-39: four exact f32 limbs (lo16, hi16) of each word."""
    w0, w1 = int(words[0]), int(words[1])
    return np.array([w0 & 0xFFFF, w0 >> 16, w1 & 0xFFFF, w1 >> 16], dtype=F32)


def decode(limbs) -> tuple[int, int]:
    """prng.rs:47-55."""
    l = [int(x) for x in np.asarray(limbs, dtype=F32)]
    return (l[0] | (l[1] << 16)) & 0xFFFFFFFF, (l[2] | (l[3] << 16)) & 0xFFFFFFFF


def _rotl(x: np.ndarray, r: int) -> np.ndarray:
    return (x << U32(r)) | (x >> U32(32 - r))


def threefry(key, c0, c1):
    """Threefry2x32 with 20 rounds (prng.rs:57-79), vectorised over counters."""
    with np.errstate(over="ignore"):
        k0, k1 = U32(key[0]), U32(key[1])
        ks = (k0, k1, U32(0x1BD11BDA) ^ k0 ^ k1)
        x0 = np.asarray(c0, dtype=U32) + ks[0]
        x1 = np.asarray(c1, dtype=U32) + ks[1]
        for rnd in range(20):
            x0 = x0 + x1
            x1 = x0 ^ _rotl(x1, ROTATIONS[rnd % 8])
            if rnd % 4 == 3:
                inj = (rnd + 1) // 4
                x0 = x0 + ks[inj % 3]
                x1 = x1 + ks[(inj + 1) % 3] + U32(inj)
    return x0, x1


def split_words(key_words, n: int) -> list[tuple[int, int]]:
    a, b = threefry(key_words, np.arange(n, dtype=U32), np.ones(n, dtype=U32))
    return [(int(a[i]), int(b[i])) for i in range(n)]


def random_key(s: int) -> np.ndarray:
    return encode(seed(s))


def random_split(key_limbs, n: int = 2) -> list[np.ndarray]:
    return [encode(w) for w in split_words(decode(key_limbs), n)]


def _bits(key_limbs, total: int):
    return threefry(decode(key_limbs), np.arange(total, dtype=U32), np.zeros(total, dtype=U32))


def uniform_from_bits(b: np.ndarray) -> np.ndarray:
    return (b >> U32(8)).astype(F32) * F32(1.0 / 16777216.0)


def normal_from_bits(b0: np.ndarray, b1: np.ndarray) -> np.ndarray:
    u1 = np.maximum(uniform_from_bits(b0), F32(1.0 / 16777216.0))
    u2 = uniform_from_bits(b1)
    radius = np.sqrt(F32(-2.0) * np.log(u1))
    theta = F32(2.0 * np.pi) * u2
    return (radius * np.cos(theta)).astype(F32)


def randint_from_bits(b0: np.ndarray, low: int, high: int) -> np.ndarray:
    u = uniform_from_bits(b0)
    v = np.floor(u * F32(high - low)) + F32(low)
    v = np.minimum(v, F32(high - 1))
    return np.maximum(v, F32(low)).astype(F32)


def random_uniform(key_limbs, shape) -> np.ndarray:
    total = int(np.prod(shape))
    b0, _ = _bits(key_limbs, total)
    return uniform_from_bits(b0).reshape(shape)


def random_normal(key_limbs, shape) -> np.ndarray:
    total = int(np.prod(shape))
    b0, b1 = _bits(key_limbs, total)
    return normal_from_bits(b0, b1).reshape(shape)


def random_randint(key_limbs, shape, low: int, high: int) -> np.ndarray:
    """Integer-valued f32 tensor (Sheaf host tensors are f32)."""
    total = int(np.prod(shape))
    b0, _ = _bits(key_limbs, total)
    return randint_from_bits(b0, low, high).reshape(shape)


def xavier_uniform(key_limbs, shape) -> np.ndarray:
    """lib/nn.shf:77-82: (u*2 - 1) * sqrt(6 / (fan_in + fan_out))."""
    limit = np.sqrt(F32(6.0) / F32(shape[0] + shape[1]))
    return ((random_uniform(key_limbs, shape) * F32(2.0) - F32(1.0)) * F32(limit)).astype(F32)
