#!/usr/bin/env python3
"""Prefill fixture from the reference engine itself (oracle/_ref, built from
sim/tmac_gguf.cpp): two seeded 64-token sequences of the batched-prefill
workload (numpy default_rng(0) token ids, as bench.py draws them) fed through
the reference's process_prompt with all four --fpga-* switches, then one greedy
step.  Saves each sequence's tokens, the hidden state after its last prompt
position, the greedy next token and its logit.  About 10 minutes of
single-threaded CPU time:

    python tests/golden/make_prefill_golden.py
"""
import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
from tmac_zynq_fpga_b200 import model  # noqa: E402

N_SEQ, LEN = 2, 64


def main():
    path = model.default_model_path(0)
    toks = np.random.default_rng(0).integers(0, model.VOCAB, size=(64, 512)).astype(np.int32)[:N_SEQ, :LEN].copy()
    R = oracle.ref()
    R.ref_decode.restype = ctypes.c_int
    R.ref_decode.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    hidden = np.zeros((N_SEQ, model.HIDDEN), np.float32)
    nxt = np.zeros(N_SEQ, np.int32)
    logit = np.zeros(N_SEQ, np.float32)
    for s in range(N_SEQ):
        prompt = np.ascontiguousarray(toks[s])
        out_t = np.zeros(1, np.int32)
        out_l = np.zeros(1, np.float32)
        out_h = np.zeros((2, model.HIDDEN), np.float32)
        n = R.ref_decode(path.encode(), prompt.ctypes.data, LEN, 1, 1, out_t.ctypes.data, out_l.ctypes.data,
                         out_h.ctypes.data)
        assert n == 1, n
        hidden[s], nxt[s], logit[s] = out_h[0], out_t[0], out_l[0]
        print("sequence", s, "next token", int(out_t[0]), flush=True)
    np.savez_compressed(os.path.join(HERE, "prefill_2x64_seed0.npz"), tokens=toks, hidden=hidden, next_token=nxt,
                        logit=logit, model_seed=np.int32(0))


if __name__ == "__main__":
    main()
