"""Host side of the FPGA's hardware-format descriptor chain (tmac_hw_desc,
vivado_integration/sw/tmac_baremetal.h:100-113): packing GGUF Q5_0 rows into
the HP FSM's 4-row tiles, writing descriptors into a DDR-image arena, and
running the chain on the GPU (tmac_chain_run_hw).

Tile layout (vivado_integration/API.md, "Q5_0 (tensor_type=1)"): 56 blocks of
48 bytes -- core 0's 22-byte GGUF block, core 1's, 4 zero bytes -- where blocks
0-27 carry rows 0 (core 0) and 2 (core 1) and blocks 28-55 rows 1 and 3, then
four UQ8.8 row norms at byte 2688 (2696 bytes per tile).  The norms are filled
as the reference's q5_preprocess_tile does (tmac_baremetal.cpp:497-528); the
GPU runner, like the reference's CPU model, recomputes them in float.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import ChainStats, _ptr, check, lib

Q8_0, Q5_0, CPU_OP = 0, 1, 15
TILE_BYTES = 2696
BLOCK_BYTES = 48
COLS = 896


def q5_0_row_norms(blocks: np.ndarray, rows: int) -> np.ndarray:
    """32767 / max|d*q| per row in float32 (1.0 for an all-zero row), as
    q5_preprocess_tile computes it (tmac_baremetal.cpp:497-516)."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(rows, COLS // 32, 22)
    d = b[:, :, 0:2].copy().view(np.float16).astype(np.float32)[..., 0]
    qh = b[:, :, 2:6].copy().view(np.uint32)[..., 0]
    qs = b[:, :, 6:22]
    wi = np.arange(32)
    ql = np.where(wi < 16, qs[:, :, wi % 16] & 0xF, qs[:, :, wi % 16] >> 4).astype(np.int32)
    hb = ((qh[:, :, None] >> wi.astype(np.uint32)) & 1).astype(np.int32)
    q = ((hb << 4) | ql) - 16
    mx = np.abs(d[:, :, None] * q.astype(np.float32)).reshape(rows, -1).max(axis=1)
    out = np.ones(rows, np.float32)
    nz = mx >= np.float32(1e-10)
    out[nz] = np.float32(32767.0) / mx[nz]
    return out


def pack_q5_0_tiles(blocks: np.ndarray, rows: int) -> np.ndarray:
    """GGUF Q5_0 rows [rows][28 blocks] -> HW tiles uint8 [ceil(rows/4)][2696]
    (rows past the end are zero blocks, as the reference pads them)."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(rows, COLS // 32, 22)
    ntiles = (rows + 3) // 4
    tiles = np.zeros((ntiles, TILE_BYTES), np.uint8)
    pad = np.zeros((ntiles * 4, COLS // 32, 22), np.uint8)
    pad[:rows] = b
    blk = tiles[:, :56 * BLOCK_BYTES].reshape(ntiles, 2, 28, BLOCK_BYTES)
    for half in range(2):           # blocks 0-27: rows 0 / 2; blocks 28-55: rows 1 / 3
        for core in range(2):
            r = np.arange(ntiles) * 4 + half + 2 * core
            blk[:, half, :, core * 22:core * 22 + 22] = pad[r]
    norms = np.ones(ntiles * 4, np.float32)
    norms[:rows] = q5_0_row_norms(b, rows)
    # uint16(ri * 256 + 0.5) as the reference writes it; it wraps for ri >= 256,
    # which is why the runner recomputes the norms
    uq = (np.floor(norms.astype(np.float64) * 256.0 + 0.5).astype(np.int64) & 0xFFFF).astype("<u2")
    tiles[:, 2688:2696] = uq.reshape(ntiles, 4).view(np.uint8)
    return tiles


def desc_bytes(next_addr=0, weight_addr=0, act_addr=0, result_addr=0, tensor_type=Q5_0, num_groups=0,
               num_tiles=1, act_total_bytes=COLS * 2) -> bytes:
    """One 32-byte descriptor, as desc_write fills it (tmac_baremetal.h:121-135)."""
    b = bytearray(32)
    b[0:4] = int(next_addr).to_bytes(4, "little")
    b[4:8] = int(weight_addr).to_bytes(4, "little")
    b[8:12] = int(act_addr).to_bytes(4, "little")
    b[12:16] = int(result_addr).to_bytes(4, "little")
    b[0x10:0x12] = int(tensor_type).to_bytes(2, "little")
    b[0x14] = num_groups & 0xFF
    b[0x16:0x18] = int(num_tiles).to_bytes(2, "little")
    b[0x18:0x1B] = int(act_total_bytes).to_bytes(3, "little")
    return bytes(b)


def chain_run_hw(arena_dev, arena_bytes, base, head, arena_host=None, max_desc=1 << 20, stream=None):
    """Runs a hardware-format chain held in a device arena (tmac_chain_run_hw)."""
    L = lib()
    f = L.tmac_chain_run_hw
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int,
                  ctypes.POINTER(ChainStats), ctypes.c_void_p]
    st = ChainStats()
    s = None if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
    check(f(_ptr(arena_dev), arena_bytes, base, _ptr(arena_host), head, max_desc, ctypes.byref(st), s))
    return st


def build_q5_0_arena(blocks: np.ndarray, rows: int, x_q: np.ndarray, base=0x10000000, num_tiles=None):
    """A DDR image holding one Q5_0 descriptor over `rows` rows (num_tiles =
    rows/4 unless given), its tiles, the int16 activations and room for the
    results.  Returns (arena uint8, head, result_addr)."""
    tiles = pack_q5_0_tiles(blocks, rows)
    nt = tiles.shape[0] if num_tiles is None else num_tiles
    head = base
    act = base + 64
    wt = act + COLS * 2
    res = (wt + tiles.nbytes + 63) // 64 * 64
    total = res + nt * 4 * 8 - base
    arena = np.zeros(total, np.uint8)
    arena[0:32] = np.frombuffer(desc_bytes(0, wt, act, res, Q5_0, 0, nt, COLS * 2), np.uint8)
    arena[act - base:act - base + COLS * 2] = np.ascontiguousarray(x_q, np.int16).view(np.uint8)
    arena[wt - base:wt - base + tiles.nbytes] = tiles.reshape(-1)
    return arena, head, res
