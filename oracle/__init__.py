"""Parity checker for the CUDA product path (test infrastructure only).

`oracle.restated` wraps liboracle.so, the C restatement of the reference's CPU
algorithm; `oracle.reference` wraps _ref/libtmac_ref.so, the reference's own
sim/ sources compiled unmodified.  Only tests/, __graft_entry__.smoke() and
bench.py's CPU baseline legs import this package; the product never does.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libtmac_ref.so")
# The reference engine with its matmul_fpga_* drivers bound to libtmac_cuda.so
# (tmac_zynq_fpga_b200/host/matmul_fpga_binding.cpp): not a checker, the
# drop-in under test.  Loading it touches no GPU; its drivers need one.
REF_SHIM_PATH = os.path.join(HERE, "_ref", "libtmac_ref_shim.so")
# The reference with only MAX_SEQ_LEN (sim/tmac_gguf.cpp:148) raised to 512, for
# decode fixtures that fill the 512-position cache (oracle/Makefile, ref512).
REF_SEQ512_PATH = os.path.join(HERE, "_ref", "libtmac_ref_seq512.so")
REF_SHIM_SEQ512_PATH = os.path.join(HERE, "_ref", "libtmac_ref_shim_seq512.so")

PATH_NATIVE, PATH_INT16, PATH_F32 = 0, 1, 2

_lib = None
_ref = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64


def build():
    """Compile liboracle.so (and _ref/ when the reference sources exist)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_quantize_x.restype = ctypes.c_float
        L.orc_quantize_x.argtypes = [_P, _I64, _P]
        L.orc_dequant.restype = ctypes.c_float
        L.orc_dequant.argtypes = [ctypes.c_int, _P, _I64, _I64, _I64]
        for n in ("orc_row_inv_q5_0", "orc_row_inv_q4_k", "orc_row_inv_q6_k"):
            getattr(L, n).argtypes = [_P, _I64, _I64, _P]
        L.orc_row_scale_q8_0.argtypes = [_P, _I64, _I64, _P, _P]
        L.orc_q8_combined_scale.restype = ctypes.c_uint16
        L.orc_q8_combined_scale.argtypes = [ctypes.c_float, ctypes.c_float]
        L.orc_units_per_row.restype = _I64
        L.orc_units_per_row.argtypes = [ctypes.c_int, ctypes.c_int, _I64]
        L.orc_gemv.restype = ctypes.c_int
        L.orc_gemv.argtypes = [ctypes.c_int, ctypes.c_int, _P, _I64, _I64, _P, _P, _P, _P, _P]
        _lib = L
    return _lib


def ref_available():
    return os.path.exists(REF_PATH)


def ref_shim(path=REF_SHIM_PATH):
    """The reference engine re-pointed at libtmac_cuda.so (see REF_SHIM_PATH;
    REF_SHIM_SEQ512_PATH for the 512-position build)."""
    R = ctypes.CDLL(path)
    R.ref_decode.restype = ctypes.c_int
    R.ref_decode.argtypes = [ctypes.c_char_p, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P]
    return R


def ref_seq512():
    """The reference engine built with a 512-position KV cache (REF_SEQ512_PATH)."""
    R = ctypes.CDLL(REF_SEQ512_PATH)
    R.ref_decode.restype = ctypes.c_int
    R.ref_decode.argtypes = [ctypes.c_char_p, _P, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, _P, _P]
    return R


def ref():
    global _ref
    if _ref is None:
        R = ctypes.CDLL(REF_PATH)
        R.ref_gemv.restype = ctypes.c_int
        R.ref_gemv.argtypes = [ctypes.c_int, ctypes.c_int, _P, _I64, _I64, ctypes.c_size_t, _P, _P, _P]
        R.ref_dequant.restype = ctypes.c_float
        R.ref_dequant.argtypes = [ctypes.c_int, _P, _I64, _I64, _I64, _I64]
        R.ref_q8_tile_sums.restype = ctypes.c_int
        R.ref_q8_tile_sums.argtypes = [_P, _I64, _I64, ctypes.c_size_t, _P, _P, _P, _P]
        R.ref_q5_0_block_sums.restype = ctypes.c_int
        R.ref_q5_0_block_sums.argtypes = [_P, _I64, _P, _P, _P]
        R.ref_q5_0_hw_tiles.restype = ctypes.c_int
        R.ref_q5_0_hw_tiles.argtypes = [_P, _I64, _I64, _P, _P, _P]
        R.ref_kquant_block_sums.restype = ctypes.c_int
        R.ref_kquant_block_sums.argtypes = [ctypes.c_int, _P, _I64, _I64, _P, _P, _P]
        _ref = R
    return _ref


class Result:
    """y plus the exact integer accumulators of one GEMV."""

    def __init__(self, y, row_acc=None, unit_acc=None):
        self.y, self.row_acc, self.unit_acc = y, row_acc, unit_acc


def gemv(qtype, w, rows, cols, x, path=PATH_NATIVE, row_max_abs=None):
    """Restated reference GEMV for one activation vector x[cols]."""
    L = lib()
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    y = np.zeros(rows, np.float32)
    units = L.orc_units_per_row(qtype, path, cols)
    row_acc = np.zeros(rows, np.int64) if path != PATH_F32 else None
    unit_acc = np.zeros((rows, units), np.int64) if units > 0 else None
    rma = None if row_max_abs is None else np.ascontiguousarray(row_max_abs, dtype=np.float32)
    rc = L.orc_gemv(qtype, path, _ptr(w), rows, cols, _ptr(x), _ptr(rma), _ptr(y),
                    _ptr(row_acc), _ptr(unit_acc))
    if rc != 0:
        raise ValueError(f"oracle rejected type={qtype} path={path} shape={rows}x{cols}")
    return Result(y, row_acc, unit_acc)


def quantize_x(x):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    xq = np.zeros(x.size, np.int16)
    xs = lib().orc_quantize_x(_ptr(x), x.size, _ptr(xq))
    return np.float32(xs), xq


def row_inv(qtype, w, rows, cols):
    L = lib()
    w = np.ascontiguousarray(w, dtype=np.uint8)
    out = np.zeros(rows, np.float32)
    fn = {6: L.orc_row_inv_q5_0, 12: L.orc_row_inv_q4_k, 14: L.orc_row_inv_q6_k}[qtype]
    fn(_ptr(w), rows, cols, _ptr(out))
    return out


def row_scale_q8(w, rows, cols, row_max_abs=None):
    out = np.zeros(rows, np.float32)
    rma = None if row_max_abs is None else np.ascontiguousarray(row_max_abs, dtype=np.float32)
    lib().orc_row_scale_q8_0(_ptr(np.ascontiguousarray(w, dtype=np.uint8)), rows, cols, _ptr(rma), _ptr(out))
    return out


# ---- the reference itself (compiled from its own sources) ----------------

def ref_gemv(qtype, w, rows, cols, x, path=PATH_NATIVE, row_max_abs=None):
    R = ref()
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    y = np.zeros(rows, np.float32)
    rma = None if row_max_abs is None else np.ascontiguousarray(row_max_abs, dtype=np.float32)
    R.ref_gemv(qtype, path, _ptr(w), rows, cols, w.nbytes, _ptr(x), _ptr(rma), _ptr(y))
    return y


def ref_unit_sums(qtype, w, rows, cols, x, row_max_abs=None):
    """The reference core models' per-unit int64 sums (see ref_harness.cpp)."""
    R = ref()
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    if qtype == 8:
        out = np.zeros((rows, (cols + 63) // 64), np.int64)
        y = np.zeros(rows, np.float32)
        rma = None if row_max_abs is None else np.ascontiguousarray(row_max_abs, dtype=np.float32)
        rc = R.ref_q8_tile_sums(_ptr(w), rows, cols, w.nbytes, _ptr(x), _ptr(rma), _ptr(y), _ptr(out))
    else:
        _, xq = quantize_x(x)  # pinned separately against the reference drivers' y
        ri = row_inv(qtype, w, rows, cols)
        if qtype == 6:
            out = np.zeros((rows, 28), np.int64)
            rc = R.ref_q5_0_block_sums(_ptr(w), rows, _ptr(xq), _ptr(ri), _ptr(out))
        else:
            out = np.zeros((rows, cols // 256), np.int64)
            rc = R.ref_kquant_block_sums(qtype, _ptr(w), rows, cols, _ptr(xq), _ptr(ri), _ptr(out))
    if rc != 0:
        raise ValueError(f"reference harness rejected type={qtype} shape={rows}x{cols} rc={rc}")
    return out


# ---- Phase-B descriptor chain ---------------------------------------------

def phaseb_run(arena, base, desc_off, cap):
    """Restated phaseb_run_descriptor: (rows, int64 accumulator[rows])."""
    L = lib()
    L.orc_phaseb_run.restype = _I64
    L.orc_phaseb_run.argtypes = [_P, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32, _P]
    arena = np.ascontiguousarray(arena, dtype=np.uint8)
    acc = np.zeros(max(cap, 1), np.int64)
    rows = L.orc_phaseb_run(_ptr(arena), base, arena.nbytes, desc_off, _ptr(acc))
    if rows < 0:
        raise ValueError("descriptor outside the arena")
    return rows, acc[:rows]


def walk_chain(arena, base, head):
    """Descriptor offsets of a chain (next_desc_addr at byte 0 of each)."""
    offs, off = [], head
    while off:
        offs.append(off)
        off = int(np.frombuffer(arena[off - base: off - base + 4].tobytes(), np.uint32)[0])
    return offs


def ref_build_chain(matmuls):
    """Builds a chain with the reference's own drivers (--fpga-phaseb) for a list of
    (type, raw blocks, rows, cols, x).  Returns (arena bytes, base, head, ys)."""
    R = ref()
    for n, res, args in (("ref_phaseb_begin", ctypes.c_int, []),
                         ("ref_phaseb_matmul", ctypes.c_int, [ctypes.c_int, _P, _I64, _I64, ctypes.c_size_t, _P, _P]),
                         ("ref_phaseb_info", ctypes.c_int, [_P, _P, _P, _P]),
                         ("ref_phaseb_copy", ctypes.c_int, [_P, ctypes.c_uint32, ctypes.c_uint32]),
                         ("ref_phaseb_run", ctypes.c_int, [ctypes.c_uint32, _P, _I64]),
                         ("ref_phaseb_verify", ctypes.c_int, [])):
        getattr(R, n).restype = res
        getattr(R, n).argtypes = args
    assert R.ref_phaseb_begin() == 0
    ys = []
    for qt, w, rows, cols, x in matmuls:
        w = np.ascontiguousarray(w, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(rows, np.float32)
        R.ref_phaseb_matmul(qt, _ptr(w), rows, cols, w.nbytes, _ptr(x), _ptr(y))
        ys.append(y)
    head, base, end, ns = (ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_int())
    R.ref_phaseb_info(ctypes.byref(head), ctypes.byref(base), ctypes.byref(end), ctypes.byref(ns))
    arena = np.zeros(end.value - base.value, np.uint8)
    assert R.ref_phaseb_copy(_ptr(arena), base.value, arena.nbytes) == 0
    return arena, base.value, head.value, ys


def ref_chain_results(arena, base, head, cap=1 << 16):
    """The reference runner's accumulators for every descriptor of a chain that
    ref_build_chain just built (phaseb_run_descriptor over the reference's DDR)."""
    R = ref()
    out = []
    for off in walk_chain(arena, base, head):
        acc = np.zeros(cap, np.int64)
        n = R.ref_phaseb_run(off, _ptr(acc), cap)
        out.append(acc[:n].copy())
    return out


def phaseb_dump_bytes(arena, base, head, desc_base, bin_base, cap=1 << 16):
    """Restated phaseb_dump_files (sim/tmac_gguf.cpp:597-708): the bytes of the
    testbench's DDR image (.bin) and header (.hdr).  The chain's descriptors are
    copied in chain order to desc_base, every next_desc_addr but the last set to
    0xFFFFFFFF; the image is DDR [bin_base, desc_base + 32 * ndesc).  The header
    is magic "PHBD", ndesc, desc_base, total rows, then per descriptor
    (result_addr, rows, act_total_bytes, previous result_addr, offset of its rows)
    as uint32 and every descriptor's int64 rows from phaseb_run.  `arena` covers
    [base, base + len) and must reach past the copied descriptors."""
    arena = np.ascontiguousarray(arena, dtype=np.uint8)
    offs = walk_chain(arena, base, head)
    n = len(offs)
    img = arena.copy()
    for i, off in enumerate(offs):
        d = arena[off - base: off - base + 32].copy()
        d[0:4] = np.frombuffer(np.uint32(0xFFFFFFFF if i < n - 1 else 0).tobytes(), np.uint8)
        img[desc_base - base + 32 * i: desc_base - base + 32 * (i + 1)] = d
    end = desc_base + 32 * n
    bin_bytes = img[bin_base - base: end - base].tobytes()
    rows, accs, table = [], [], []
    prev, pos = 0, 0
    for off in offs:
        r, acc = phaseb_run(arena, base, off, cap)
        d = arena[off - base: off - base + 32]
        result_addr = int(np.frombuffer(d[12:16].tobytes(), np.uint32)[0])
        act_bytes = int(d[0x17]) | (int(d[0x18]) << 8)
        table.append((result_addr, r, act_bytes, prev, pos))
        accs.append(acc)
        pos += r
        prev = result_addr
    hdr = np.array([0x50484244, n, desc_base, pos], np.uint32).tobytes()
    hdr += np.array(table, np.uint32).reshape(-1).tobytes() if table else b""
    hdr += b"".join(a.astype(np.int64).tobytes() for a in accs)
    return bin_bytes, hdr
