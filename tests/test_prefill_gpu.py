"""Batched prefill (tmac_model_prefill) against the decode engine and the reference.

Prefill runs n_seq sequences through all layers at once on the tensor cores;
every per-token operation is the decode engine's, so each position's hidden
state must equal the decode engine's after feeding the same tokens up to that
position, bit for bit.  The decode engine itself matches the reference's
greedy tokens (test_decode_gpu.py), so the first generated token after the
fixture prompt must also be the reference's.
"""
import os

import numpy as np
import pytest

import tmac_zynq_fpga_b200 as tm
from tmac_zynq_fpga_b200 import model

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = os.path.join(HERE, "golden", "decode_greedy_seed0.npz")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mdl():
    m = tm.Model(model.default_model_path(0), switches=tm.SW_ALL, max_seq=512)
    yield m
    m.free()


def test_prefill_matches_decode_every_position(mdl):
    g = np.load(FIX)
    prompt = g["prompt"].astype(np.int32)
    other = model.prompt_tokens(len(prompt), seed=5)
    nxt, hid = mdl.prefill(np.stack([prompt, other]), want_hidden=True)
    for p in range(len(prompt)):
        _, h = mdl.generate(prompt[:p + 1], 0, want_hidden=True)
        np.testing.assert_array_equal(hid[0, p], h[0], err_msg=f"position {p}")
    toks, _ = mdl.generate(other, 1)
    assert nxt[1] == toks[0]
    assert nxt[0] == g["tokens"][0]  # the reference's first greedy token


def test_prefill_sequences_are_independent(mdl):
    a = model.prompt_tokens(24, seed=11)
    b = model.prompt_tokens(24, seed=12)
    n2, h2 = mdl.prefill(np.stack([a, b]), want_hidden=True)
    n1, h1 = mdl.prefill(b[None, :], want_hidden=True)
    assert n2[1] == n1[0]
    np.testing.assert_array_equal(h2[1], h1[0])


def test_prefill_growing_batches_keep_weight_planes(mdl):
    """A larger batch re-makes the activation buffers; the cached weight planes
    (the Q8_0 attn_v layers) must survive it."""
    a = model.prompt_tokens(16, seed=21)
    n_small, h_small = mdl.prefill(a[None, :], want_hidden=True)
    batch = np.stack([model.prompt_tokens(16, seed=22 + i) for i in range(5)] + [a])
    n_big, h_big = mdl.prefill(batch, want_hidden=True)
    assert n_big[-1] == n_small[0]
    np.testing.assert_array_equal(h_big[-1], h_small[0])


def test_prefill_long_odd_length_matches_decode(mdl):
    """131 tokens: two K/V tiles of 128 positions, a last query block of 3 and
    score rows padded to a multiple of 4."""
    a = model.prompt_tokens(131, seed=31)
    nxt, hid = mdl.prefill(a[None, :], want_hidden=True)
    for p in (0, 63, 64, 127, 128, 130):
        _, h = mdl.generate(a[:p + 1], 0, want_hidden=True)
        np.testing.assert_array_equal(hid[0, p], h[0], err_msg=f"position {p}")
    toks, _ = mdl.generate(a, 1)
    assert nxt[0] == toks[0]


def test_prefill_64x512_matches_decode_at_full_size():
    """The benchmark's batched prefill, 64 sequences x 512 seeded tokens (M =
    32768 rows per projection): for three sequences, the hidden states at
    positions 0, 255 and 511 equal the decode engine's after feeding the same
    tokens (bit for bit), and so does the greedy next token."""
    m = tm.Model(model.default_model_path(0), switches=tm.SW_ALL, max_seq=513)
    try:
        toks = np.random.default_rng(0).integers(0, model.VOCAB, size=(64, 512)).astype(np.int32)
        nxt, hid = m.prefill(toks, want_hidden=True)
        for s in (0, 31, 63):
            for p in (0, 255):
                _, h = m.generate(toks[s, :p + 1], 0, want_hidden=True)
                np.testing.assert_array_equal(hid[s, p].view(np.int32), h[0].view(np.int32),
                                              err_msg=f"sequence {s} position {p}")
            t, h = m.generate(toks[s], 1, want_hidden=True)
            np.testing.assert_array_equal(hid[s, 511].view(np.int32), h[0].view(np.int32),
                                          err_msg=f"sequence {s} position 511")
            assert nxt[s] == t[0], f"sequence {s}"
    finally:
        m.free()


PREFILL_FIX = os.path.join(HERE, "golden", "prefill_2x64_seed0.npz")
HIDDEN_RTOL = 5e-4  # as test_decode_gpu.py: the context ops' expf/logf against glibc


@pytest.mark.skipif(not os.path.exists(PREFILL_FIX), reason="prefill fixture missing")
def test_prefill_matches_reference_process_prompt(mdl):
    """Two 64-token sequences of the benchmark's prefill workload against the
    reference engine's own process_prompt + one greedy step (fixture from
    oracle/_ref, tests/golden/make_prefill_golden.py): the hidden state after
    the last prompt position within HIDDEN_RTOL, the next token identical."""
    g = np.load(PREFILL_FIX)
    toks = g["tokens"]
    nxt, hid = mdl.prefill(toks, want_hidden=True)
    for s in range(len(toks)):
        ref = g["hidden"][s]
        err = np.abs(hid[s, -1] - ref).max() / np.abs(ref).max()
        assert err < HIDDEN_RTOL, f"sequence {s}: relative hidden error {err:.3g}"
        assert nxt[s] == g["next_token"][s], f"sequence {s}"
