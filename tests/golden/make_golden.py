#!/usr/bin/env python3
"""Generates the golden fixtures in this directory from the reference itself:
liuwantao3/tmac-zynq-fpga sim/tmac_gguf.cpp + sim/fpga_sim.hpp compiled
unmodified into oracle/_ref/libtmac_ref.so (oracle/Makefile).  Run from the
repository root after `make -C oracle`:

    python tests/golden/make_golden.py           # GEMV fixtures
    python tests/golden/make_golden.py --chain   # Phase-B chain fixture

Each fixture holds seeded synthetic GGUF blocks, the activations, and the
reference's outputs: y for the FPGA-model path (matmul_fpga_*), the INT16
fallback and the FP32 path, plus the core models' per-unit int64 sums.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from tmac_zynq_fpga_b200 import synth  # noqa: E402

CASES = [
    # name, type, rows, cols, seed
    ("q5_0_16x896", synth.Q5_0, 16, 896, 1),
    ("q8_0_70x896", synth.Q8_0, 70, 896, 2),
    ("q8_0_33x96", synth.Q8_0, 33, 96, 3),
    ("q4_k_12x512", synth.Q4_K, 12, 512, 4),
    ("q6_k_12x512", synth.Q6_K, 12, 512, 5),
]


def main():
    if not oracle.ref_available():
        sys.exit("oracle/_ref/libtmac_ref.so missing: run `make -C oracle` with the reference sources present")
    for name, qt, rows, cols, seed in CASES:
        w = synth.make_weights(qt, rows, cols, seed=seed)
        x = synth.make_activations(cols, seed=seed)[0]
        out = {"type": np.int32(qt), "rows": np.int64(rows), "cols": np.int64(cols), "w": w, "x": x}
        out["y_native"] = oracle.ref_gemv(qt, w, rows, cols, x, path=oracle.PATH_NATIVE)
        out["y_int16"] = oracle.ref_gemv(qt, w, rows, cols, x, path=oracle.PATH_INT16)
        out["y_f32"] = oracle.ref_gemv(qt, w, rows, cols, x, path=oracle.PATH_F32)
        out["unit_acc"] = oracle.ref_unit_sums(qt, w, rows, cols, x)
        if qt == synth.Q8_0:
            rma = np.abs(np.random.default_rng(seed).normal(0, 0.02, rows)).astype(np.float32) * 4
            out["row_max_abs"] = rma
            out["y_native_rma"] = oracle.ref_gemv(qt, w, rows, cols, x, path=oracle.PATH_NATIVE, row_max_abs=rma)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
        print("wrote", name)


if __name__ == "__main__" and "--chain" not in sys.argv:
    main()


def make_chain_fixture():
    """A Phase-B chain built by the reference's own drivers with --fpga-phaseb
    (Q5_0 128x896, Q4_K 112x512, Q6_K 64x512), its DDR arena image and the
    reference runner's int64 accumulators per descriptor."""
    ms = [(synth.Q5_0, synth.make_weights(synth.Q5_0, 128, 896, seed=61), 128, 896,
           synth.make_activations(896, seed=61)[0]),
          (synth.Q4_K, synth.make_weights(synth.Q4_K, 112, 512, seed=62), 112, 512,
           synth.make_activations(512, seed=62)[0]),
          (synth.Q6_K, synth.make_weights(synth.Q6_K, 64, 512, seed=63), 64, 512,
           synth.make_activations(512, seed=63)[0])]
    arena, base, head, ys = oracle.ref_build_chain(ms)
    res = oracle.ref_chain_results(arena, base, head)
    np.savez_compressed(os.path.join(HERE, "phaseb_chain.npz"), arena=arena, base=np.uint32(base),
                        head=np.uint32(head), offsets=np.array(oracle.walk_chain(arena, base, head), np.uint32),
                        results=np.concatenate(res), counts=np.array([len(r) for r in res], np.int64))
    print("wrote phaseb_chain")


if __name__ == "__main__" and "--chain" in sys.argv:
    make_chain_fixture()
