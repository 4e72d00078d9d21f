"""Hardware-format descriptor chain (tmac_hw_desc, vivado_integration/sw/
tmac_baremetal.h:100-113; tiles per vivado_integration/API.md "Q5_0
(tensor_type=1)").

CPU: the tile packer against the reference's own HP-FSM core model
(axi_vecmul_tile_q5_0_4x896_axilite, sim/fpga_sim.hpp:1194-1249, in
oracle/_ref) -- its int64 rows on packed tiles equal the oracle's Q5_0 rows --
and descriptor validation of tmac_chain_run_hw (refused before any device
access when walked from the host mirror).
GPU: one num_tiles=224 descriptor over the 896x896 attn_q matrix, and a
chain mixing Q5_0, CPU_OP passthrough and an (unsupported) Q8_0 descriptor;
every int64 row identical to the oracle's.
"""
import ctypes

import numpy as np
import pytest

import oracle
import tmac_zynq_fpga_b200 as tm
from tmac_zynq_fpga_b200 import hwchain, synth

needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


def _case(rows, seed):
    w = synth.make_weights(synth.Q5_0, rows, 896, seed=seed)
    x = synth.make_activations(896, seed=seed)[0]
    _, xq = oracle.quantize_x(x)
    return w, x, xq


def test_row_norms_equal_oracle_row_inv():
    w, _, _ = _case(64, 5)
    ri = oracle.row_inv(synth.Q5_0, w, 64, 896)
    np.testing.assert_array_equal(hwchain.q5_0_row_norms(w, 64).view(np.int32), ri.view(np.int32))


@needs_ref
@pytest.mark.parametrize("rows", [896, 6])
def test_packed_tiles_through_reference_core_model(rows):
    w, x, xq = _case(rows, 0 if rows == 896 else 9)
    tiles = hwchain.pack_q5_0_tiles(w, rows)
    nt = tiles.shape[0]
    norms = np.ones(nt * 4, np.float32)
    norms[:rows] = hwchain.q5_0_row_norms(w, rows)
    out = np.zeros(nt * 4, np.int64)
    R = oracle.ref()
    assert R.ref_q5_0_hw_tiles(tiles.ctypes.data, nt, hwchain.TILE_BYTES, xq.ctypes.data, norms.ctypes.data,
                               out.ctypes.data) == 0
    o = oracle.gemv(synth.Q5_0, w, rows, 896, x)
    np.testing.assert_array_equal(out[:rows], o.row_acc)
    assert not out[rows:].any()


def test_desc_bytes_layout():
    d = hwchain.desc_bytes(0x100, 0x200, 0x300, 0x400, hwchain.Q5_0, 3, 224, 0x012345)
    assert d[0:4] == (0x100).to_bytes(4, "little") and d[12:16] == (0x400).to_bytes(4, "little")
    assert d[0x10:0x12] == b"\x01\x00" and d[0x14] == 3 and d[0x16:0x18] == (224).to_bytes(2, "little")
    assert d[0x18:0x1B] == b"\x45\x23\x01" and d[0x1B:] == b"\x00" * 5


@pytest.mark.parametrize("case", ["weights_out", "act_short", "result_out", "cycle", "head_out", "cpu_op_overlap"])
def test_hw_chain_validation_rejects_bad_descriptors(case):
    base, n = 0x1000, 8192
    arena = bytearray(n)
    head = base
    d = {"weights_out": hwchain.desc_bytes(0, base + 64, base + 64, base + 64, hwchain.Q5_0, 0, 4),
         "act_short": hwchain.desc_bytes(0, base + 64, base + 64, base + 64, hwchain.Q5_0, 0, 1, 1790),
         "result_out": hwchain.desc_bytes(0, base + 64, base + 64, base + n - 16, hwchain.Q5_0, 0, 1),
         "cycle": hwchain.desc_bytes(base, base + 64, base + 64, base + 64, hwchain.CPU_OP, 0, 1, 0),
         "head_out": None,
         "cpu_op_overlap": hwchain.desc_bytes(0, 0, base + 64, base + 96, hwchain.CPU_OP, 0, 1, 64)}[case]
    if d is None:
        head = base + n
    else:
        arena[0:32] = d
    host = np.frombuffer(bytes(arena), np.uint8)
    st = tm.ChainStats()
    f = tm.lib().tmac_chain_run_hw
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int,
                  ctypes.POINTER(tm.ChainStats), ctypes.c_void_p]
    rc = f(1, n, base, host.ctypes.data, head, 64, ctypes.byref(st), None)
    assert rc == -4, (case, rc, tm.lib().tmac_last_error())


@pytest.mark.gpu
@pytest.mark.parametrize("mirror", [True, False])
def test_gpu_hw_q5_0_descriptor_224_tiles(mirror):
    """attn_q 896x896 as one num_tiles=224 descriptor."""
    torch = pytest.importorskip("torch")
    w, x, xq = _case(896, 0)
    arena, head, res = hwchain.build_q5_0_arena(w, 896, xq)
    base = head
    dev = torch.from_numpy(arena.copy()).cuda()
    st = hwchain.chain_run_hw(dev, arena.nbytes, base, head, arena_host=arena if mirror else None)
    torch.cuda.synchronize()
    assert st.descriptors == 1 and st.unsupported == 0 and st.result_rows == 896
    got = np.frombuffer(dev.cpu().numpy()[res - base:res - base + 896 * 8].tobytes(), np.int64)
    np.testing.assert_array_equal(got, oracle.gemv(synth.Q5_0, w, 896, 896, x).row_acc)
    assert tm.device_error(0) == 0


@pytest.mark.gpu
def test_gpu_hw_chain_mixed_descriptors():
    """Q5_0 (ragged: 10 rows in 3 tiles) -> CPU_OP passthrough -> Q8_0 (skipped)
    -> Q5_0 with num_tiles = 0 (one tile)."""
    torch = pytest.importorskip("torch")
    base = 0x20000000
    w1, x1, xq1 = _case(10, 21)
    w2, x2, xq2 = _case(4, 22)
    t1, t2 = hwchain.pack_q5_0_tiles(w1, 10), hwchain.pack_q5_0_tiles(w2, 4)
    lay = {"d0": 0, "d1": 32, "d2": 64, "d3": 96, "a1": 128, "a2": 128 + 1792, "w1": 4096,
           "w2": 4096 + t1.nbytes, "r1": 16384, "r2": 16384 + 12 * 8, "cp": 17408, "q8w": 18432}
    A = {k: base + v for k, v in lay.items()}
    arena = np.zeros(20480, np.uint8)

    def put(off, b):
        arena[off - base:off - base + len(b)] = np.frombuffer(bytes(b), np.uint8)
    put(A["d0"], hwchain.desc_bytes(A["d1"], A["w1"], A["a1"], A["r1"], hwchain.Q5_0, 0, 3, 1792))
    put(A["d1"], hwchain.desc_bytes(A["d2"], 0, A["a2"], A["cp"], hwchain.CPU_OP, 0, 1, 256))
    put(A["d2"], hwchain.desc_bytes(A["d3"], A["q8w"], A["a1"], A["q8w"], hwchain.Q8_0, 14, 1, 1792))
    put(A["d3"], hwchain.desc_bytes(0, A["w2"], A["a2"], A["r2"], hwchain.Q5_0, 0, 0, 1792))
    put(A["a1"], xq1.view(np.uint8))
    put(A["a2"], xq2.view(np.uint8))
    put(A["w1"], t1.reshape(-1))
    put(A["w2"], t2.reshape(-1))
    dev = torch.from_numpy(arena.copy()).cuda()
    st = hwchain.chain_run_hw(dev, arena.nbytes, base, A["d0"], arena_host=arena)
    torch.cuda.synchronize()
    assert st.descriptors == 4 and st.unsupported == 1 and st.result_rows == 12 + 4
    out = dev.cpu().numpy()
    r1 = np.frombuffer(out[lay["r1"]:lay["r1"] + 12 * 8].tobytes(), np.int64)
    np.testing.assert_array_equal(r1[:10], oracle.gemv(synth.Q5_0, w1, 10, 896, x1).row_acc)
    assert not r1[10:].any()
    r2 = np.frombuffer(out[lay["r2"]:lay["r2"] + 4 * 8].tobytes(), np.int64)
    np.testing.assert_array_equal(r2, oracle.gemv(synth.Q5_0, w2, 4, 896, x2).row_acc)
    assert out[lay["cp"]:lay["cp"] + 256].tobytes() == arena[lay["a2"]:lay["a2"] + 256].tobytes()
    assert out[lay["q8w"]:lay["q8w"] + 64].tobytes() == arena[lay["q8w"]:lay["q8w"] + 64].tobytes()
