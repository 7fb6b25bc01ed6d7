"""nanoGPT token sampling, restated from the reference (test-only).

generate-token (examples/nanogpt/model.shf:116-125):
    logits     = gpt-forward(ids, params)           ; the full window
    last-logit = last(reshape(logits, [-1, V])) / temp
    [vals idx] = top_k(last-logit, min(top-k, V))
    probs      = softmax(vals)
    [new-key subkey] = random-split(key)
    next-id    = idx[choice(subkey, len(probs), :p probs)]
choice (sheaf/src/lowering/stablehlo/random_ops.rs:164-180):
    u = uniform(subkey, []); cumsum = tril(ones[k, k]) @ probs;
    index = min(k - count(cumsum > u), k - 1)
and the window update slide-window (sample.shf:28-29, append-and-roll):
drop the first id, append the new one.

Sampling arithmetic is float32 throughout: the temperature-scaled logits,
the softmax (max-subtracted exp, sequential sum) and the sequential cumsum.
top_k orders by value, descending, ties by ascending index.
"""
from __future__ import annotations

import numpy as np

from . import prng

F32 = np.float32


def top_k(x, k: int):
    """Stable descending order: (values, indices) of the k largest."""
    x = np.asarray(x, F32)
    order = np.argsort(-x, kind="stable")[:k]
    return x[order], order


def softmax_f32(v):
    """lib/nn.shf:24-26 in float32: exp(v - max) / sum, summed in order."""
    v = np.asarray(v, F32)
    e = np.exp(v - v.max()).astype(F32)
    s = F32(0.0)
    for x in e:
        s = F32(s + x)
    return (e / s).astype(F32)


def choice_index(subkey_limbs, probs):
    """random_ops.rs:164-180. Returns (index, margin): margin is the distance
    of u to the nearest cumsum value (a float32 rounding difference can only
    change the index when it is tiny)."""
    probs = np.asarray(probs, F32)
    k = len(probs)
    u = F32(prng.random_uniform(subkey_limbs, ()))
    c = F32(0.0)
    cumsum = np.empty(k, F32)
    for i, p in enumerate(probs):
        c = F32(c + p)
        cumsum[i] = c
    count = int(np.sum(cumsum > u))
    return min(k - count, k - 1), float(np.min(np.abs(cumsum.astype(np.float64) - float(u))))


def generate_token(last_logits, key_limbs, k: int, temp: float):
    """One step of model.shf:116-125 from the last position's logits.
    Returns (next_id, new_key_limbs, margin)."""
    x = (np.asarray(last_logits, F32) / F32(temp)).astype(F32)
    vals, idx = top_k(x, min(k, len(x)))
    probs = softmax_f32(vals)
    new_key, subkey = prng.random_split(key_limbs, 2)
    i, margin = choice_index(subkey, probs)
    return int(idx[i]), new_key, margin


def slide_window(ids, token):
    """append-and-roll: drop the oldest id, append the new one."""
    ids = np.asarray(ids, F32)
    return np.concatenate([ids[1:], np.array([token], F32)])
