"""tmac_zynq_fpga_b200 -- B200 (sm_100a) replacement for the FPGA quantized-GEMV
cores of liuwantao3/tmac-zynq-fpga.

The product is libtmac_cuda.so (C ABI in include/tmac_cuda.h, CUDA kernels in
csrc/).  This module binds it with ctypes and mirrors the reference's host
interface for the hot path (sim/tmac_gguf.cpp:466-493):

* ``Tensor``                         -- the reference's Tensor record (:163-169)
* ``matmul_fpga_q8 / _q5_0 / _q4_k / _q6_k / _int16(A, x, y, rows, cols)``
* ``matmul(A, x, y, rows, cols)``    -- the dispatch switch, driven by ``switches``
* ``Weight``                          -- a registered device-resident weight

There is no CPU fallback: if the library or a B200 is missing, calls raise.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

from . import synth  # noqa: F401  (seeded synthetic inputs)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtmac_cuda.so")
HEADER = os.path.join(HERE, "..", "include", "tmac_cuda.h")

F32, F16, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 6, 8, 12, 14
MODE_NATIVE, MODE_INT16, MODE_F32 = 0, 1, 2

STATUS = {0: "TMAC_OK", -1: "TMAC_ERR_INVALID", -2: "TMAC_ERR_TYPE", -3: "TMAC_ERR_SHAPE",
          -4: "TMAC_ERR_BOUNDS", -5: "TMAC_ERR_CUDA", -6: "TMAC_ERR_NCCL", -7: "TMAC_ERR_TIMEOUT",
          -8: "TMAC_ERR_NOMEM", -9: "TMAC_ERR_NODEV"}


class TmacError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


class ChainStats(ctypes.Structure):
    """tmac_chain_stats"""
    _fields_ = [("descriptors", ctypes.c_int), ("unsupported", ctypes.c_int), ("result_rows", ctypes.c_int64)]


_lib = None
_P = ctypes.c_void_p
_I64 = ctypes.c_int64


def build(force=False):
    """Compile libtmac_cuda.so in-tree (nvcc, sm_100a)."""
    from . import buildlib as _b
    return _b.build(force=force)


def lib():
    """The loaded libtmac_cuda.so (built on first use when nvcc is present)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        sig = {
            "tmac_abi_version": (ctypes.c_int, []),
            "tmac_last_error": (ctypes.c_char_p, []),
            "tmac_device_error": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
            "tmac_weight_register": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, _I64, _I64, _P, ctypes.c_size_t,
                                                    ctypes.c_int, _P, ctypes.c_int, ctypes.POINTER(_P)]),
            "tmac_weight_free": (ctypes.c_int, [_P]),
            "tmac_weight_info": (ctypes.c_int, [_P, _P, _P, _P, _P, _P]),
            "tmac_weight_device_bytes": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_size_t)]),
            "tmac_weight_row_norm": (ctypes.c_int, [_P, _P]),
            "tmac_units_per_row": (_I64, [ctypes.c_int, ctypes.c_int, _I64]),
            "tmac_gemv": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, _P]),
            "tmac_gemv_acc": (ctypes.c_int, [_P, _P, _P, _P, _P, ctypes.c_int, _P]),
            "tmac_gemv_q8_0": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, _P]),
            "tmac_gemv_q5_0": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, _P]),
            "tmac_gemv_q4_k": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, _P]),
            "tmac_gemv_q6_k": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, _P]),
            "tmac_gemv_int16": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, _P]),
            "tmac_gemv_host": (ctypes.c_int, [_P, _P, _P, ctypes.c_int]),
            "tmac_gemv_static": (ctypes.c_int, [_P, _P, _P, ctypes.c_int, _P]),
            "tmac_gemm": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int, _P]),
            "tmac_xchg_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_P)]),
            "tmac_xchg_ipc_handle": (ctypes.c_int, [_P, _P]),
            "tmac_xchg_open": (ctypes.c_int, [_P, ctypes.c_char_p]),
            "tmac_xchg_top1": (ctypes.c_int, [_P, _P, _P]),
            "tmac_set_pdl": (ctypes.c_int, [ctypes.c_int]),
            "tmac_phaseb_dump": (ctypes.c_int, [_P, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                                ctypes.c_uint32, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]),
            "tmac_xchg_gemv_top1": (ctypes.c_int, [_P, _P, _P, _P, _P, ctypes.c_int64, _P]),
            "tmac_xchg_free": (ctypes.c_int, [_P]),
            "tmac_reserve": (ctypes.c_int, [ctypes.c_int, _I64, _I64]),
            "tmac_top1": (ctypes.c_int, [_P, _I64, _I64, _P, _P]),
            "tmac_gemv_top1": (ctypes.c_int, [_P, _P, _P, _P, _I64, ctypes.c_int, _P]),
            "tmac_top1_decode": (ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_float),
                                                ctypes.POINTER(_I64)]),
            "tmac_quantize_x": (ctypes.c_int, [_P, _I64, ctypes.c_int, _P, _P, _P]),
            "tmac_gemv_xq": (ctypes.c_int, [_P, _P, _P, _P, ctypes.c_int, _P]),
            "tmac_chain_run": (ctypes.c_int, [_P, ctypes.c_size_t, ctypes.c_uint32, _P, ctypes.c_uint32,
                                              ctypes.c_int, ctypes.POINTER(ChainStats), _P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc):
    if rc != 0:
        raise TmacError(rc, lib().tmac_last_error().decode(errors="replace"))
    return rc


def _ptr(a):
    """Address of a numpy array, a torch tensor, an int, or None."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()  # torch.Tensor


def device_error(device=0):
    code = ctypes.c_int(0)
    check(lib().tmac_device_error(device, ctypes.byref(code)))
    return code.value


def units_per_row(qtype, mode, cols):
    return lib().tmac_units_per_row(qtype, mode, cols)


class Weight:
    """A weight tensor registered on one device (see tmac_weight_register)."""

    def __init__(self, qtype, rows, cols, blocks, mode=MODE_NATIVE, row_max_abs=None, device=0):
        self.qtype, self.rows, self.cols, self.mode, self.device = qtype, rows, cols, mode, device
        h = _P()
        on_dev = 0
        if isinstance(blocks, np.ndarray):
            blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
            nbytes = blocks.nbytes
        elif isinstance(blocks, (bytes, bytearray)):
            blocks = np.frombuffer(blocks, dtype=np.uint8)
            nbytes = blocks.nbytes
        else:  # torch tensor on device
            on_dev = 1 if blocks.is_cuda else 0
            nbytes = blocks.numel() * blocks.element_size()
        rma = None if row_max_abs is None else np.ascontiguousarray(row_max_abs, dtype=np.float32)
        check(lib().tmac_weight_register(qtype, mode, rows, cols, _ptr(blocks), nbytes, on_dev, _ptr(rma), device,
                                         ctypes.byref(h)))
        self.handle = h.value
        self.units = units_per_row(qtype, mode, cols)

    def free(self):
        if getattr(self, "handle", None):
            lib().tmac_weight_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def device_bytes(self):
        n = ctypes.c_size_t(0)
        check(lib().tmac_weight_device_bytes(self.handle, ctypes.byref(n)))
        return n.value

    def row_norm(self):
        out = np.zeros(self.rows, np.float32)
        check(lib().tmac_weight_row_norm(self.handle, _ptr(out)))
        return out

    def gemv(self, x, y, batch=1, stream=None, row_acc=None, unit_acc=None):
        """Device GEMV on torch tensors / device pointers (asynchronous)."""
        s = None if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
        check(lib().tmac_gemv_acc(self.handle, _ptr(x), _ptr(y), _ptr(row_acc), _ptr(unit_acc), batch, s))

    def gemm(self, x, y, m, row_acc=None, stream=None):
        """Tensor-core batched matmul: y[m][rows] for m fp32 activation rows (device)."""
        s = None if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
        check(lib().tmac_gemm(self.handle, _ptr(x), _ptr(y), _ptr(row_acc), m, s))

    def gemv_top1(self, x, y, key, index_base=0, batch=1, stream=None):
        """y = W.x plus the packed top-1 key of y (device uint64/int64 key[batch])."""
        s = None if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
        check(lib().tmac_gemv_top1(self.handle, _ptr(x), _ptr(y), _ptr(key), index_base, batch, s))

    def gemv_host(self, x, batch=None):
        """Host-buffer GEMV: numpy x[batch][cols] -> numpy y[batch][rows] (synchronous)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if batch is None:
            batch = x.size // self.cols
        y = np.empty((batch, self.rows), np.float32)
        check(lib().tmac_gemv_host(self.handle, _ptr(x), _ptr(y), batch))
        return y


# ---------------------------------------------------------------------------
# Mirror of the reference's host interface for the hot path.

@dataclass
class Tensor:
    """sim/tmac_gguf.cpp:163-169: name, rows, cols, GGUF type, raw block bytes."""
    name: str
    rows: int
    cols: int
    type: int
    data: np.ndarray

    @property
    def n_bytes(self):
        return int(self.data.nbytes)


@dataclass
class Switches:
    """The reference's dispatch flags (tmac_gguf.cpp:178-183, set by argv at :2084-2091)."""
    use_fpga: bool = False
    fpga_q8: bool = False
    fpga_q4k: bool = False
    fpga_q5_0: bool = False
    fpga_q6_k: bool = False
    fpga_phaseb: bool = False

    def parse(self, argv):
        for a in argv:
            if a in ("--fpga", "--fpga-int16"):
                self.use_fpga = True
            elif a == "--fpga-q8":
                self.use_fpga = self.fpga_q8 = True
            elif a == "--fpga-q4k":
                self.use_fpga = self.fpga_q4k = True
            elif a == "--fpga-q5-0":
                self.use_fpga = self.fpga_q5_0 = True
            elif a == "--fpga-q6-k":
                self.use_fpga = self.fpga_q6_k = True
            elif a == "--fpga-phaseb":
                self.fpga_phaseb = self.use_fpga = True
                self.fpga_q5_0 = self.fpga_q6_k = self.fpga_q4k = self.fpga_q8 = True
        return self


switches = Switches()
_cache: dict = {}


def _weight_for(A: Tensor, mode: int, row_max_abs=None, device=0) -> Weight:
    key = (id(A.data), A.data.ctypes.data, A.rows, A.cols, A.type, mode,
           None if row_max_abs is None else row_max_abs.ctypes.data, device)
    w = _cache.get(key)
    if w is None:
        w = Weight(A.type, A.rows, A.cols, A.data, mode=mode, row_max_abs=row_max_abs, device=device)
        _cache[key] = w
    return w


def _run(A, x, y, rows, cols, mode, row_max_abs=None):
    if rows != A.rows or cols != A.cols:
        raise TmacError(-3, f"rows/cols {rows}x{cols} do not match tensor {A.rows}x{A.cols}")
    out = _weight_for(A, mode, row_max_abs).gemv_host(np.asarray(x, np.float32).reshape(1, cols), 1)
    y[:rows] = out[0]


def matmul_fpga_q8(A, x, y, rows, cols, row_max_abs=None):
    """tmac_gguf.cpp:948 -- Q8_0 core path (row_max_abs: optional per-row table)."""
    if A.type != Q8_0:
        raise TmacError(-2, "matmul_fpga_q8 needs a Q8_0 tensor")
    _run(A, x, y, rows, cols, MODE_NATIVE, row_max_abs)


def matmul_fpga_q5_0(A, x, y, rows, cols):
    """tmac_gguf.cpp:1221 -- Q5_0 core path."""
    if A.type != Q5_0:
        raise TmacError(-2, "matmul_fpga_q5_0 needs a Q5_0 tensor")
    _run(A, x, y, rows, cols, MODE_NATIVE)


def matmul_fpga_q4_k(A, x, y, rows, cols):
    """tmac_gguf.cpp:1097 -- Q4_K core path."""
    if A.type != Q4_K:
        raise TmacError(-2, "matmul_fpga_q4_k needs a Q4_K tensor")
    _run(A, x, y, rows, cols, MODE_NATIVE)


def matmul_fpga_q6_k(A, x, y, rows, cols):
    """tmac_gguf.cpp:1367 -- Q6_K core path."""
    if A.type != Q6_K:
        raise TmacError(-2, "matmul_fpga_q6_k needs a Q6_K tensor")
    _run(A, x, y, rows, cols, MODE_NATIVE)


def matmul_fpga_int16(A, x, y, rows, cols):
    """tmac_gguf.cpp:887 -- INT16 fallback core path (any type)."""
    _run(A, x, y, rows, cols, MODE_INT16)


def matmul(A, x, y, rows, cols, sw: Switches | None = None):
    """tmac_gguf.cpp:473-493 -- route by type and switches; no switch = FP32 path."""
    sw = sw or switches
    if sw.use_fpga:
        if sw.fpga_q5_0 and A.type == Q5_0:
            return matmul_fpga_q5_0(A, x, y, rows, cols)
        if sw.fpga_q6_k and A.type == Q6_K:
            return matmul_fpga_q6_k(A, x, y, rows, cols)
        if sw.fpga_q4k and A.type == Q4_K:
            return matmul_fpga_q4_k(A, x, y, rows, cols)
        if sw.fpga_q8 and A.type == Q8_0:
            return matmul_fpga_q8(A, x, y, rows, cols)
        return matmul_fpga_int16(A, x, y, rows, cols)
    _run(A, x, y, rows, cols, MODE_F32)


def chain_run(arena_dev, arena_bytes, base, head, arena_host=None, max_desc=1 << 20, stream=None):
    """Replays a Phase-B descriptor chain held in a device arena (tmac_chain_run);
    the int64 results land at each descriptor's result_addr inside the arena."""
    st = ChainStats()
    s = None if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
    check(lib().tmac_chain_run(_ptr(arena_dev), arena_bytes, base, _ptr(arena_host), head, max_desc,
                               ctypes.byref(st), s))
    return st


def phaseb_dump(arena_host, base, head, desc_base, bin_base, bin_path, hdr_path, device=0):
    """Writes the reference's --dump-phaseb testbench files for a chain held in the
    host DDR image `arena_host` (tmac_phaseb_dump; expected rows from the GPU)."""
    arena_host = np.ascontiguousarray(arena_host, dtype=np.uint8)
    check(lib().tmac_phaseb_dump(_ptr(arena_host), arena_host.nbytes, base, head, desc_base, bin_base,
                                 os.fsencode(bin_path), os.fsencode(hdr_path), device))


def top1_decode(key):
    """(value, index) of a packed top-1 key."""
    v, i = ctypes.c_float(), _I64()
    check(lib().tmac_top1_decode(ctypes.c_uint64(int(key) & 0xFFFFFFFFFFFFFFFF), ctypes.byref(v), ctypes.byref(i)))
    return v.value, i.value


# ---------------------------------------------------------------------------
# Whole-model greedy decode (tmac_model_*).

SW_FPGA, SW_Q8, SW_Q5_0, SW_Q4_K, SW_Q6_K, SW_ALL = 1, 2, 4, 8, 16, 31


def switches_from_argv(argv):
    """The reference's --fpga-* flags as a TMAC_SW_* bit mask."""
    sw = Switches().parse(argv)
    bits = SW_FPGA if sw.use_fpga else 0
    bits |= (SW_Q8 if sw.fpga_q8 else 0) | (SW_Q5_0 if sw.fpga_q5_0 else 0)
    bits |= (SW_Q4_K if sw.fpga_q4k else 0) | (SW_Q6_K if sw.fpga_q6_k else 0)
    return bits


class Model:
    """A device-resident Qwen2-0.5B-shaped model loaded from a `.tmac` file."""

    def __init__(self, path, switches=SW_ALL, max_seq=512, device=0):
        L = lib()
        for n, args in (("tmac_model_create", [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_P)]),
                        ("tmac_model_load_tmac", [_P, ctypes.c_char_p]), ("tmac_model_finalize", [_P]),
                        ("tmac_model_reset", [_P, _P]), ("tmac_model_forward", [_P, ctypes.c_int, ctypes.c_int, _P]),
                        ("tmac_model_prefill", [_P, _P, ctypes.c_int, ctypes.c_int, _P, _P, _P]),
                        ("tmac_model_logits", [_P, _P]), ("tmac_model_buffers", [_P, _P, _P, _P]),
                        ("tmac_model_generate", [_P, _P, ctypes.c_int, ctypes.c_int, _P, _P, _P]),
                        ("tmac_model_decode_engine", [_P]), ("tmac_model_free", [_P])):
            getattr(L, n).restype = ctypes.c_int
            getattr(L, n).argtypes = args
        h = _P()
        check(L.tmac_model_create(device, switches, max_seq, ctypes.byref(h)))
        self.handle = h.value
        check(L.tmac_model_load_tmac(self.handle, path.encode()))
        check(L.tmac_model_finalize(self.handle))

    def generate(self, prompt, n_gen, want_hidden=False, stream=None):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        toks = np.zeros(n_gen, np.int32)
        hid = np.zeros((n_gen + 1, 896), np.float32) if want_hidden else None
        s = None if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
        check(lib().tmac_model_generate(self.handle, prompt.ctypes.data, len(prompt), n_gen, toks.ctypes.data,
                                        None if hid is None else hid.ctypes.data, s))
        return toks, hid

    def decode_engine(self):
        """1: the last generate ran the persistent decode kernel; 0: the per-kernel
        engine; -1: no generate yet."""
        return lib().tmac_model_decode_engine(self.handle)

    def prefill(self, tokens, want_hidden=False, stream=None):
        """Batched prefill of tokens [n_seq][len]: (next greedy token per sequence,
        hidden states [n_seq][len][896] or None)."""
        tokens = np.ascontiguousarray(np.atleast_2d(tokens), dtype=np.int32)
        n_seq, ln = tokens.shape
        nxt = np.zeros(n_seq, np.int32)
        hid = np.zeros((n_seq, ln, 896), np.float32) if want_hidden else None
        s = None if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
        check(lib().tmac_model_prefill(self.handle, tokens.ctypes.data, n_seq, ln, nxt.ctypes.data,
                                       None if hid is None else hid.ctypes.data, s))
        return nxt, hid

    def free(self):
        if getattr(self, "handle", None):
            lib().tmac_model_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
