"""nanoGPT's data path restated (test-only): get-batch of
examples/nanogpt/train.shf:15-21 over the reference's PRNG (oracle.prng).

    starts = random-randint key [batch] 0 (len(data) - block - 1)
    idx    = starts[:, None] + arange(block)[None, :]
    x, y   = data[idx], data[idx + 1]
"""
from __future__ import annotations

import numpy as np

from . import prng


def get_batch(data, key_limbs, block: int, batch: int):
    data = np.asarray(data, np.float32)
    starts = prng.random_randint(key_limbs, (batch,), 0, len(data) - block - 1).astype(np.int64)
    idx = starts[:, None] + np.arange(block)[None, :]
    return data[idx], data[idx + 1], starts
