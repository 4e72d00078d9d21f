"""The C-ABI library loads and exports every function include/*.h declares
(no GPU needed: nothing is called that touches a device)."""
import ctypes
import glob
import os
import re

import tmac_zynq_fpga_b200 as tm

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(tmac_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("tmac_weight_register", "tmac_gemv", "tmac_gemv_q8_0", "tmac_gemv_q5_0", "tmac_gemv_q4_k",
              "tmac_gemv_q6_k", "tmac_gemv_int16", "tmac_gemv_host", "tmac_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    L = tm.lib()
    missing = [n for n in sorted(declared_functions()) if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_abi_version_and_error_string():
    L = tm.lib()
    assert L.tmac_abi_version() == 1
    assert isinstance(L.tmac_last_error(), bytes)


def test_units_per_row_matches_reference_tiling():
    assert tm.units_per_row(tm.Q8_0, tm.MODE_NATIVE, 896) == 14      # 64-column tiles
    assert tm.units_per_row(tm.Q5_0, tm.MODE_NATIVE, 896) == 28      # 32-column blocks
    assert tm.units_per_row(tm.Q4_K, tm.MODE_NATIVE, 4864) == 19     # 256-column blocks
    assert tm.units_per_row(tm.Q6_K, tm.MODE_NATIVE, 4864) == 19
    assert tm.units_per_row(tm.Q5_0, tm.MODE_INT16, 896) == 14
    assert tm.units_per_row(tm.Q5_0, tm.MODE_F32, 896) == 0


def test_registration_rejects_bad_arguments_without_gpu():
    L = tm.lib()
    h = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * 64)()
    # bad type / shape / size checks come before any device access
    assert L.tmac_weight_register(99, 0, 1, 32, buf, 64, 0, None, 0, ctypes.byref(h)) == -2
    assert L.tmac_weight_register(tm.Q5_0, 0, 1, 33, buf, 64, 0, None, 0, ctypes.byref(h)) == -3
    assert L.tmac_weight_register(tm.Q5_0, 0, 4, 32, buf, 64, 0, None, 0, ctypes.byref(h)) == -4
    assert L.tmac_weight_register(tm.F32, 0, 4, 4, buf, 64, 0, None, 0, ctypes.byref(h)) == -2
    assert b"n_bytes" in L.tmac_last_error() or L.tmac_last_error()


def test_peer_exchange_rejects_bad_arguments_without_gpu():
    L = tm.lib()
    key = ctypes.c_uint64(0)
    out = ctypes.c_void_p()
    # argument checks come before any device access
    assert L.tmac_xchg_create(0, 0, 0, ctypes.byref(out)) != 0        # world < 1
    assert L.tmac_xchg_create(0, 2, 2, ctypes.byref(out)) != 0        # rank >= world
    assert L.tmac_xchg_create(0, 2, 0, None) != 0
    assert L.tmac_xchg_top1(None, ctypes.byref(key), None) != 0
    assert L.tmac_xchg_gemv_top1(None, None, None, None, None, 0, None) != 0
    assert L.tmac_xchg_ipc_handle(None, None) != 0
    assert L.tmac_xchg_open(None, None) != 0
    assert L.tmac_xchg_free(None) == 0


def test_pdl_switch_returns_previous_setting():
    L = tm.lib()
    prev = L.tmac_set_pdl(1)
    assert L.tmac_set_pdl(0) == 1
    assert L.tmac_set_pdl(prev) == 0
