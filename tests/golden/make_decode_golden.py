#!/usr/bin/env python3
"""Greedy-decode fixture from the reference engine itself (oracle/_ref, built
from sim/tmac_gguf.cpp): the seed-0 synthetic Qwen2-0.5B-shaped model
(tmac_zynq_fpga_b200.model, deterministic), an 8-token seeded prompt, 64 greedy
steps with all four --fpga-* switches.  Saves the tokens, each chosen token's
logit and the hidden state after the prompt and after every step.
About 4-5 minutes of single-threaded CPU time:

    python tests/golden/make_decode_golden.py [n_gen]

With --pos512 it makes decode_greedy_seed0_pos512.npz instead: a 448-token
seeded prompt and 64 greedy steps, so the KV cache fills all 512 positions of
the decode configuration.  The reference's cache stops at MAX_SEQ_LEN = 256
(sim/tmac_gguf.cpp:148), so this run uses oracle/_ref/libtmac_ref_seq512.so,
the reference compiled with only that constant set to 512
(make -C oracle ref512 REF=<reference tree>).  Hidden states are kept after the
prompt and after every step.  About 35 minutes of single-threaded CPU time.
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
from tmac_zynq_fpga_b200 import model  # noqa: E402


def main(n_gen=64, n_prompt=8, lib=None, out="decode_greedy_seed0.npz"):
    path = model.default_model_path(0)
    prompt = model.prompt_tokens(n_prompt, seed=0)
    R = oracle.ref_seq512() if lib == "seq512" else oracle.ref()
    R.ref_decode.restype = ctypes.c_int
    R.ref_decode.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    toks = np.zeros(n_gen, np.int32)
    logit = np.zeros(n_gen, np.float32)
    hidden = np.zeros((n_gen + 1, model.HIDDEN), np.float32)
    n = R.ref_decode(path.encode(), prompt.ctypes.data, len(prompt), n_gen, 1, toks.ctypes.data,
                     logit.ctypes.data, hidden.ctypes.data)
    assert n == n_gen, n
    np.savez_compressed(os.path.join(HERE, out), prompt=prompt, tokens=toks,
                        logit=logit, hidden=hidden, model_seed=np.int32(0))
    print("tokens", toks.tolist())


if __name__ == "__main__":
    if "--pos512" in sys.argv:
        main(64, 448, "seq512", "decode_greedy_seed0_pos512.npz")
    else:
        main(int(sys.argv[1]) if len(sys.argv) > 1 else 64)
