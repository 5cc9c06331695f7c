"""Seeded GGUF weight rows for the projection tests: random quant bytes with
finite, moderate f16 scales in each block's scale fields."""
import numpy as np

from oracle import oracle as orc

BLOCK = {orc.QTYPE_Q4_K: (256, 144), orc.QTYPE_Q6_K: (256, 210), orc.QTYPE_Q4_0: (32, 18),
         orc.QTYPE_Q8_0: (32, 34), orc.QTYPE_F16: (1, 2)}


def random_rows(qtype, rows, cols, seed):
    rng = np.random.default_rng(seed)
    if qtype == orc.QTYPE_F16:
        return rng.standard_normal((rows, cols)).astype(np.float16).view(np.uint8).reshape(rows, -1)
    unit, nb = BLOCK[qtype]
    blocks = rng.integers(0, 256, (rows * cols // unit, nb), dtype=np.uint8)

    def put_f16(col, lo, hi):
        v = rng.uniform(lo, hi, blocks.shape[0]).astype(np.float16).view(np.uint8)
        blocks[:, col:col + 2] = v.reshape(-1, 2)

    if qtype == orc.QTYPE_Q4_K:
        put_f16(0, 0.001, 0.02)   # d
        put_f16(2, 0.001, 0.02)   # dmin
    elif qtype == orc.QTYPE_Q6_K:
        put_f16(208, 0.001, 0.02)
    else:
        put_f16(0, 0.001, 0.05)
    return blocks.reshape(rows, -1)
