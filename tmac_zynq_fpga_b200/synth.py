"""Seeded synthetic GGUF blocks and activations in the shapes and value
distributions of the benchmark configurations.

The real Qwen2-0.5B GGUF is not available, so weights are random-init with the
block layouts the reference decodes (sim/fpga_sim.hpp:503-525,
sim/tmac_gguf.cpp:225-393):

* Q8_0  34 B / 32 values: fp16 d, 32 x int8
* Q5_0  22 B / 32 values: fp16 d, u32 qh (high bits), 16 B qs (nibbles j, j+16)
* Q4_K 144 B / 256 values: fp16 d, fp16 dmin, 12 B packed 6-bit scales/mins, 128 B qs
* Q6_K 210 B / 256 values: 128 B ql, 64 B qh, 16 x int8 scales, fp16 d

Distributions: Q5_0 d = |N(0,0.02)|/16; Q8_0 d = |N(0,0.02)|/127 with quants
uniform in [-127, 127]; Q4_K d, dmin = |N(0,0.02)|/64 with uniform scale and
quant bytes; Q6_K d = |N(0,0.02)|/32 with int8 sub-scales uniform in [-32, 31];
activations N(0, 1).  All from numpy.random.default_rng(seed).
"""
from __future__ import annotations

import numpy as np

F32, F16, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 6, 8, 12, 14

BLOCK_VALUES = {Q8_0: 32, Q5_0: 32, Q4_K: 256, Q6_K: 256}
BLOCK_BYTES = {Q8_0: 34, Q5_0: 22, Q4_K: 144, Q6_K: 210}
TYPE_NAMES = {F32: "F32", F16: "F16", Q5_0: "Q5_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}


def tensor_nbytes(qtype: int, rows: int, cols: int) -> int:
    if qtype == F32:
        return rows * cols * 4
    if qtype == F16:
        return rows * cols * 2
    return rows * (cols // BLOCK_VALUES[qtype]) * BLOCK_BYTES[qtype]


def _f16_bits(v: np.ndarray) -> np.ndarray:
    return np.asarray(v, dtype=np.float32).astype(np.float16).view(np.uint16)


def make_weights(qtype: int, rows: int, cols: int, seed: int = 0) -> np.ndarray:
    """Raw GGUF block bytes (uint8, row-major blocks) for a rows x cols tensor."""
    rng = np.random.default_rng(seed)
    if qtype in (F32, F16):
        w = rng.normal(0.0, 0.02, size=(rows, cols)).astype(np.float32)
        return (w if qtype == F32 else w.astype(np.float16)).view(np.uint8).reshape(-1)
    nv, nb = BLOCK_VALUES[qtype], BLOCK_BYTES[qtype]
    if cols % nv:
        raise ValueError(f"cols={cols} is not a multiple of the {TYPE_NAMES[qtype]} block ({nv})")
    n = rows * (cols // nv)
    blk = np.zeros((n, nb), dtype=np.uint8)
    if qtype == Q8_0:
        d = _f16_bits(np.abs(rng.normal(0.0, 0.02, n)) / 127.0)
        blk[:, 0:2] = d.view(np.uint8).reshape(n, 2)
        blk[:, 2:34] = rng.integers(-127, 128, size=(n, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    elif qtype == Q5_0:
        d = _f16_bits(np.abs(rng.normal(0.0, 0.02, n)) / 16.0)
        blk[:, 0:2] = d.view(np.uint8).reshape(n, 2)
        blk[:, 2:6] = rng.integers(0, 1 << 32, size=n, dtype=np.uint64).astype(np.uint32).view(np.uint8).reshape(n, 4)
        blk[:, 6:22] = rng.integers(0, 256, size=(n, 16), dtype=np.uint8)
    elif qtype == Q4_K:
        d = _f16_bits(np.abs(rng.normal(0.0, 0.02, n)) / 64.0)
        dmin = _f16_bits(np.abs(rng.normal(0.0, 0.02, n)) / 64.0)
        blk[:, 0:2] = d.view(np.uint8).reshape(n, 2)
        blk[:, 2:4] = dmin.view(np.uint8).reshape(n, 2)
        blk[:, 4:144] = rng.integers(0, 256, size=(n, 140), dtype=np.uint8)
    elif qtype == Q6_K:
        blk[:, 0:192] = rng.integers(0, 256, size=(n, 192), dtype=np.uint8)
        blk[:, 192:208] = rng.integers(-32, 32, size=(n, 16), dtype=np.int16).astype(np.int8).view(np.uint8)
        d = _f16_bits(np.abs(rng.normal(0.0, 0.02, n)) / 32.0)
        blk[:, 208:210] = d.view(np.uint8).reshape(n, 2)
    else:
        raise ValueError(f"unsupported type {qtype}")
    return blk.reshape(-1)


def make_activations(cols: int, batch: int = 1, seed: int = 0) -> np.ndarray:
    """fp32 activations ~N(0,1), shape [batch, cols]."""
    rng = np.random.default_rng(seed + 0x5EED)
    return rng.standard_normal((batch, cols), dtype=np.float32)
