"""Phase-B descriptor chain (fpga_sim.hpp:1254-1310, tmac_gguf.cpp:513-880).

CPU: the restated runner (oracle) against the fixture the reference's own
chain builder and runner produced, and against the compiled reference on a
fresh chain; descriptor validation of tmac_chain_run (no device access when
the chain is walked from a host mirror and rejected).
GPU: tmac_chain_run on the same arena images; every int64 result identical.
"""
import ctypes
import os

import numpy as np
import pytest

import oracle
import tmac_zynq_fpga_b200 as tm
from tmac_zynq_fpga_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = os.path.join(HERE, "golden", "phaseb_chain.npz")
needs_ref = pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")


def load_fixture():
    g = np.load(FIX)
    return g["arena"], int(g["base"]), int(g["head"]), list(g["offsets"]), g["results"], g["counts"]


def test_fixture_descriptors_match_reference_layout():
    arena, base, head, offs, _, counts = load_fixture()
    assert oracle.walk_chain(arena, base, head) == [int(o) for o in offs]
    d = np.frombuffer(arena[offs[0] - base: offs[0] - base + 32].tobytes(), dtype=np.uint8)
    assert d[0x14] == 6 and d[0x15] == 8  # Q5_0, 8-row tiles
    assert int.from_bytes(d[0x12:0x14].tobytes(), "little") == 4944  # TMAC_PHASEB_Q5_0_TILE_BYTES
    assert list(counts) == [128, 112, 64]


def test_oracle_chain_matches_fixture():
    arena, base, head, offs, results, counts = load_fixture()
    pos = 0
    for off, n in zip(offs, counts):
        rows, acc = oracle.phaseb_run(arena, base, int(off), 4096)
        assert rows == n
        np.testing.assert_array_equal(acc, results[pos:pos + n])
        pos += n


@needs_ref
def test_oracle_chain_matches_reference_fresh_chain():
    ms = [(synth.Q6_K, synth.make_weights(synth.Q6_K, 96, 768, seed=71), 96, 768,
           synth.make_activations(768, seed=71)[0] * 3),
          (synth.Q5_0, synth.make_weights(synth.Q5_0, 24, 896, seed=72), 24, 896,
           synth.make_activations(896, seed=72)[0]),
          (synth.Q4_K, synth.make_weights(synth.Q4_K, 56, 1024, seed=73), 56, 1024,
           synth.make_activations(1024, seed=73)[0])]
    arena, base, head, _ = oracle.ref_build_chain(ms)
    for off, ref in zip(oracle.walk_chain(arena, base, head), oracle.ref_chain_results(arena, base, head)):
        rows, acc = oracle.phaseb_run(arena, base, off, 4096)
        np.testing.assert_array_equal(acc, ref)


def _desc(next_off=0, wt=0, act=0, res=0, ntiles=1, tb=4944, typ=6, tr=8, cg=1):
    b = bytearray(32)
    b[0:4] = next_off.to_bytes(4, "little")
    b[4:8] = wt.to_bytes(4, "little")
    b[8:12] = act.to_bytes(4, "little")
    b[12:16] = res.to_bytes(4, "little")
    b[0x10:0x12] = ntiles.to_bytes(2, "little")
    b[0x12:0x14] = tb.to_bytes(2, "little")
    b[0x14], b[0x15], b[0x19] = typ, tr, cg
    return bytes(b)


@pytest.mark.parametrize("case", ["weights_out", "result_out", "cycle", "head_out", "cg_zero", "q5_rows"])
def test_chain_validation_rejects_bad_descriptors(case):
    """Rejected before any device access (walked from the host mirror)."""
    base, n = 0x1000, 4096
    arena = bytearray(n)
    d = {"weights_out": _desc(wt=base + 100, act=base + 100, res=base),
         "result_out": _desc(wt=base + 64, act=base + 64, res=base + n - 8, ntiles=0),
         "cycle": _desc(next_off=base, wt=base + 64, act=base + 64, res=base + 64, ntiles=0),
         "head_out": None,
         "cg_zero": _desc(typ=12, tb=8288, tr=56, cg=0),
         "q5_rows": _desc(tr=4)}[case]
    head = base
    if d is None:
        head = base + n
    else:
        arena[0:32] = d
        if case == "result_out":
            arena[0:32] = _desc(wt=base + 64, act=base + 64, res=base + n - 8, ntiles=1)
    host = np.frombuffer(bytes(arena), np.uint8)
    st = tm.ChainStats()
    rc = tm.lib().tmac_chain_run(1, n, base, host.ctypes.data, head, 64, ctypes.byref(st), None)
    assert rc == -4, (case, rc, tm.lib().tmac_last_error())


@pytest.mark.gpu
@pytest.mark.parametrize("mirror", [True, False])
def test_gpu_chain_matches_fixture(mirror):
    torch = pytest.importorskip("torch")
    arena, base, head, offs, results, counts = load_fixture()
    dev = torch.from_numpy(arena.copy()).cuda()
    st = tm.chain_run(dev, arena.nbytes, base, head, arena_host=arena if mirror else None)
    torch.cuda.synchronize()
    assert st.descriptors == 3 and st.unsupported == 0 and st.result_rows == int(counts.sum())
    out = dev.cpu().numpy()
    pos = 0
    for off, n in zip(offs, counts):
        d = arena[off - base: off - base + 32]
        res = int.from_bytes(d[12:16].tobytes(), "little")
        got = np.frombuffer(out[res - base: res - base + 8 * n].tobytes(), np.int64)
        np.testing.assert_array_equal(got, results[pos:pos + n])
        pos += n


@pytest.mark.gpu
@needs_ref
def test_gpu_chain_full_model_shapes():
    """Config-scale chain: attn_q 896x896 and ffn_gate 4864x896 Q5_0, ffn_down
    896x4864 as Q4_K and Q6_K, built by the reference's drivers; GPU results
    equal the reference runner's, descriptor by descriptor."""
    torch = pytest.importorskip("torch")
    ms = [(synth.Q5_0, synth.make_weights(synth.Q5_0, 896, 896, seed=81), 896, 896,
           synth.make_activations(896, seed=81)[0]),
          (synth.Q5_0, synth.make_weights(synth.Q5_0, 4864, 896, seed=82), 4864, 896,
           synth.make_activations(896, seed=82)[0]),
          (synth.Q4_K, synth.make_weights(synth.Q4_K, 896, 4864, seed=83), 896, 4864,
           synth.make_activations(4864, seed=83)[0]),
          (synth.Q6_K, synth.make_weights(synth.Q6_K, 896, 4864, seed=84), 896, 4864,
           synth.make_activations(4864, seed=84)[0])]
    arena, base, head, _ = oracle.ref_build_chain(ms)
    refs = oracle.ref_chain_results(arena, base, head, cap=8192)
    dev = torch.from_numpy(arena.copy()).cuda()
    tm.chain_run(dev, arena.nbytes, base, head, arena_host=arena)
    torch.cuda.synchronize()
    out = dev.cpu().numpy()
    for off, ref in zip(oracle.walk_chain(arena, base, head), refs):
        res = int.from_bytes(arena[off - base + 12: off - base + 16].tobytes(), "little")
        got = np.frombuffer(out[res - base: res - base + 8 * len(ref)].tobytes(), np.int64)
        np.testing.assert_array_equal(got, ref)


# ---- Phase-B dump (phaseb_dump_files, tmac_gguf.cpp:597-708) ---------------

def _dump_case():
    arena, base, head, offs, results, counts = load_fixture()
    desc_base = base + ((arena.nbytes + 31) & ~31)       # the reference: next free offset rounded to 32
    room = np.concatenate([arena, np.zeros(desc_base - base - arena.nbytes + 32 * len(offs), np.uint8)])
    return room, base, head, offs, results, counts, desc_base


def test_oracle_dump_layout_and_rows():
    room, base, head, offs, results, counts, desc_base = _dump_case()
    b, h = oracle.phaseb_dump_bytes(room, base, head, desc_base, base)
    hdr = np.frombuffer(h[:16], np.uint32)
    assert list(hdr) == [0x50484244, len(offs), desc_base, int(sum(counts))]
    table = np.frombuffer(h[16:16 + 20 * len(offs)], np.uint32).reshape(-1, 5)
    assert list(table[:, 1]) == list(counts) and list(table[:, 4]) == [0, 128, 240]
    assert table[0, 3] == 0 and list(table[1:, 3]) == list(table[:-1, 0])
    np.testing.assert_array_equal(np.frombuffer(h[16 + 20 * len(offs):], np.int64), results)
    assert len(b) == desc_base + 32 * len(offs) - base
    nxt = [int(np.frombuffer(b[desc_base - base + 32 * i: desc_base - base + 32 * i + 4], np.uint32)[0])
           for i in range(len(offs))]
    assert nxt == [0xFFFFFFFF] * (len(offs) - 1) + [0]
    for i, off in enumerate(offs):  # every other descriptor byte copied unchanged
        assert b[desc_base - base + 32 * i + 4: desc_base - base + 32 * (i + 1)] == \
            room[off - base + 4: off - base + 32].tobytes()


def test_dump_rejects_bad_arguments_without_gpu():
    room, base, head, offs, *_ , desc_base = _dump_case()
    L = tm.lib()
    buf = np.ascontiguousarray(room)
    assert L.tmac_phaseb_dump(None, 0, base, head, desc_base, base, b"a", b"b", 0) == -1
    # misaligned or too-late desc_base, bin_base past desc_base: refused before any device access
    assert L.tmac_phaseb_dump(buf.ctypes.data, buf.nbytes, base, head, desc_base + 4, base, b"a", b"b", 0) == -4
    assert L.tmac_phaseb_dump(buf.ctypes.data, buf.nbytes, base, head, desc_base + 64, base, b"a", b"b", 0) == -4
    assert L.tmac_phaseb_dump(buf.ctypes.data, buf.nbytes, base, head, desc_base, desc_base + 32, b"a", b"b", 0) == -4


@pytest.mark.gpu
def test_gpu_dump_files_equal_the_oracle():
    room, base, head, offs, results, counts, desc_base = _dump_case()
    out = os.path.join(HERE, ".phaseb_out")
    os.makedirs(out, exist_ok=True)
    bp, hp = os.path.join(out, "tb_phaseb.bin"), os.path.join(out, "tb_phaseb.hdr")
    tm.phaseb_dump(room, base, head, desc_base, base, bp, hp)
    b, h = oracle.phaseb_dump_bytes(room, base, head, desc_base, base)
    assert open(bp, "rb").read() == b
    assert open(hp, "rb").read() == h


@needs_ref
def test_dump_format_equals_the_reference_dump_files():
    """The Phase-B testbench files written by the reference's own
    phaseb_dump_files (tmac_gguf.cpp:597-708, run through oracle/_ref; it writes
    fixed /tmp paths) are byte-identical to the oracle's restatement, which the
    GPU test above pins tmac_phaseb_dump to.  Covers the 20-byte header entries
    (the code, not the 24 its comment states) and the DDR image."""
    ms = [(synth.Q5_0, synth.make_weights(synth.Q5_0, 16, 896, seed=61), 16, 896,
           synth.make_activations(896, seed=61)[0]),
          (synth.Q6_K, synth.make_weights(synth.Q6_K, 64, 512, seed=62), 64, 512,
           synth.make_activations(512, seed=62)[0]),
          (synth.Q4_K, synth.make_weights(synth.Q4_K, 56, 256, seed=63), 56, 256,
           synth.make_activations(256, seed=63)[0])]
    arena, base, head, _ = oracle.ref_build_chain(ms)
    ndesc = len(oracle.walk_chain(arena, base, head))
    desc_base = (base + arena.nbytes + 31) & ~31
    room = np.concatenate([arena, np.zeros(desc_base - base - arena.nbytes + 32 * ndesc, np.uint8)])
    b, h = oracle.phaseb_dump_bytes(room, base, head, desc_base, base)
    R = oracle.ref()
    R.ref_phaseb_dump.restype = ctypes.c_int
    assert R.ref_phaseb_dump() == 0
    assert open("/tmp/tb_phaseb.bin", "rb").read() == b
    assert open("/tmp/tb_phaseb.hdr", "rb").read() == h
