"""Qwen2-0.5B-shaped model files in the reference's `.tmac` format, with seeded
random-init weights (the real GGUF is not available).

`.tmac` layout (scripts/extract_tmac.py:1-23, read by load_tmac,
sim/tmac_gguf.cpp:1894-1947): b"TMAC", u64 n_tensors, then per tensor
u64 name_len, name bytes, u64 rows, u64 cols, u32 GGUF type, u64 n_bytes, data.
rows = GGUF ne[1] (output dim), cols = ne[0] (input dim).

Quantisation mix of the benchmark model: layers {0,1,3,6,7,8,9,10,13,16,19,21} use
Q8_0 attn_v and Q6_K ffn_down, the other 12 layers Q5_0 attn_v and Q4_K
ffn_down; attn_q/k/output and ffn_gate/up are Q5_0; token_embd is Q8_0 (tied
with the output); norms are F32 ~ 1 + N(0, 0.02); q/k/v biases F32 ~ N(0, 0.02).
"""
from __future__ import annotations

import os
import struct

import numpy as np

from . import synth

HIDDEN, INTER, VOCAB, LAYERS = 896, 4864, 151936, 24
HEADS, KV_HEADS, HEAD_DIM = 14, 2, 64
KV_DIM = KV_HEADS * HEAD_DIM
Q8_LAYERS = {0, 1, 3, 6, 7, 8, 9, 10, 13, 16, 19, 21}


def tensor_list(layers: int = LAYERS):
    """(name, rows, cols, type) of every tensor, in file order."""
    out = [("token_embd.weight", VOCAB, HIDDEN, synth.Q8_0), ("output_norm.weight", HIDDEN, 1, synth.F32)]
    for l in range(layers):
        p = f"blk.{l}."
        q8 = l in Q8_LAYERS
        out += [
            (p + "attn_norm.weight", HIDDEN, 1, synth.F32),
            (p + "attn_q.weight", HIDDEN, HIDDEN, synth.Q5_0),
            (p + "attn_q.bias", HIDDEN, 1, synth.F32),
            (p + "attn_k.weight", KV_DIM, HIDDEN, synth.Q5_0),
            (p + "attn_k.bias", KV_DIM, 1, synth.F32),
            (p + "attn_v.weight", KV_DIM, HIDDEN, synth.Q8_0 if q8 else synth.Q5_0),
            (p + "attn_v.bias", KV_DIM, 1, synth.F32),
            (p + "attn_output.weight", HIDDEN, HIDDEN, synth.Q5_0),
            (p + "ffn_norm.weight", HIDDEN, 1, synth.F32),
            (p + "ffn_gate.weight", INTER, HIDDEN, synth.Q5_0),
            (p + "ffn_up.weight", INTER, HIDDEN, synth.Q5_0),
            (p + "ffn_down.weight", HIDDEN, INTER, synth.Q6_K if q8 else synth.Q4_K),
        ]
    return out


def make_tensor(name, rows, cols, qtype, seed):
    rng = np.random.default_rng(seed)
    if qtype == synth.F32:
        if name.endswith("norm.weight"):
            v = 1.0 + rng.normal(0.0, 0.02, rows)
        else:
            v = rng.normal(0.0, 0.02, rows)
        return v.astype(np.float32).view(np.uint8)
    return synth.make_weights(qtype, rows, cols, seed=seed)


def write_tmac(path: str, seed: int = 0, layers: int = LAYERS):
    """Writes a seeded random-init model; returns the path."""
    tl = tensor_list(layers)
    with open(path, "wb") as f:
        f.write(b"TMAC")
        f.write(struct.pack("<Q", len(tl)))
        for i, (name, rows, cols, qtype) in enumerate(tl):
            data = make_tensor(name, rows, cols, qtype, seed * 100003 + i)
            nb = name.encode()
            f.write(struct.pack("<Q", len(nb)))
            f.write(nb)
            f.write(struct.pack("<QQIQ", rows, cols, qtype, data.nbytes))
            f.write(data.tobytes())
    return path


def read_tmac(path: str):
    """{name: (rows, cols, type, uint8 data)} of a `.tmac` file (load_tmac's reader)."""
    out = {}
    with open(path, "rb") as f:
        if f.read(4) != b"TMAC":
            raise ValueError("not a .tmac file")
        (n,) = struct.unpack("<Q", f.read(8))
        for _ in range(n):
            (ln,) = struct.unpack("<Q", f.read(8))
            name = f.read(ln).decode()
            rows, cols, qtype, nb = struct.unpack("<QQIQ", f.read(28))
            out[name] = (rows, cols, qtype, np.frombuffer(f.read(nb), dtype=np.uint8))
    return out


def default_model_path(seed: int = 0) -> str:
    """Cached synthetic model under ~/.cache (regenerated when missing)."""
    d = os.path.join(os.path.expanduser("~"), ".cache", "tmac_b200")
    os.makedirs(d, exist_ok=True)
    p = os.path.join(d, f"qwen2_0_5b_synth_seed{seed}.tmac")
    if not os.path.exists(p):
        tmp = f"{p}.tmp{os.getpid()}"  # one writer per process; the rename is atomic
        write_tmac(tmp, seed=seed)
        os.replace(tmp, p)
    return p


def prompt_tokens(n: int = 8, seed: int = 0):
    rng = np.random.default_rng(seed + 777)
    return rng.integers(0, VOCAB, size=n).astype(np.int32)
