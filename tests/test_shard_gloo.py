"""Vocab-sharded logits top-1 on 2 CPU ranks (gloo): each rank computes its
shard of a Q8_0 logits GEMV with the oracle, packs its shard's top-1 key, and a
MAX all-reduce must give the global greedy token (lowest index on ties)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from tmac_zynq_fpga_b200 import shard, synth

ROWS, COLS = 2048, 896


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, tie, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = synth.make_weights(synth.Q8_0, ROWS, COLS, seed=5)
    x = synth.make_activations(COLS, seed=5)[0]
    r0, r1 = shard.shard_bounds(ROWS, world, rank)
    part = w[r0 * 28 * 34: r1 * 28 * 34]
    y = oracle.gemv(synth.Q8_0, part, r1 - r0, COLS, x).y
    if tie:  # the same maximum in both shards: the lower global index must win
        y[:] = -1.0
        y[7] = 3.0
    key = torch.tensor([int(shard.pack_keys(y, r0).max())], dtype=torch.int64)
    shard.all_reduce_top1(key)
    out[rank] = int(key.item())
    dist.destroy_process_group()


@pytest.mark.parametrize("tie", [False, True])
def test_two_rank_top1_matches_global_argmax(tie):
    world = 2
    out = mp.Manager().dict()
    mp.spawn(_rank_main, args=(world, _free_port(), tie, out), nprocs=world, join=True)
    w = synth.make_weights(synth.Q8_0, ROWS, COLS, seed=5)
    x = synth.make_activations(COLS, seed=5)[0]
    y = oracle.gemv(synth.Q8_0, w, ROWS, COLS, x).y
    want = 7 if tie else shard.top1_index(y)
    for r in range(world):
        val, idx = shard.unpack_key(out[r])
        assert idx == want
        if not tie:
            assert np.float32(val) == y[want]


def test_key_order_and_roundtrip():
    y = np.array([-2.0, -0.0, 0.0, 1.5, -np.inf, np.inf, 1.5, 3.25e-30], np.float32)
    k = shard.pack_keys(y, 100)
    assert (k >= 0).all()
    order = np.argsort(-k, kind="stable")
    assert order[0] == 5 and shard.unpack_key(k[5]) == (np.inf, 105)
    assert k[3] > k[6]  # equal values: the lower index has the larger key
    for i, v in enumerate(y):
        val, idx = shard.unpack_key(k[i])
        assert idx == 100 + i and np.float32(val).tobytes() == v.tobytes()


def test_shard_bounds_cover_vocab():
    for world in (1, 2, 4, 8):
        b = [shard.shard_bounds(151936, world, r) for r in range(world)]
        assert b[0][0] == 0 and b[-1][1] == 151936
        assert all(b[i][1] == b[i + 1][0] for i in range(world - 1))


def _prefill_rank(rank, world, port, n_seq, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    toks = np.random.default_rng(3).integers(0, 151936, size=(n_seq, 16))
    s0, s1 = shard.sequence_shard(n_seq, world, rank)
    # stand-in for each rank's prefill: a deterministic function of the sequence
    local = (toks[s0:s1].sum(axis=1) * 7919 % 151936).astype(np.int32)
    out[rank] = shard.gather_next_tokens(local, n_seq).tolist()
    dist.destroy_process_group()


@pytest.mark.parametrize("n_seq", [64, 7])
def test_two_rank_sequence_sharded_prefill_gathers_in_batch_order(n_seq):
    world = 2
    out = mp.Manager().dict()
    mp.spawn(_prefill_rank, args=(world, _free_port(), n_seq, out), nprocs=world, join=True)
    toks = np.random.default_rng(3).integers(0, 151936, size=(n_seq, 16))
    expect = (toks.sum(axis=1) * 7919 % 151936).astype(np.int32).tolist()
    assert out[0] == expect and out[1] == expect


def _logits_rank(rank, world, port, rows, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    w = synth.make_weights(synth.Q8_0, rows, COLS, seed=9)
    x = synth.make_activations(COLS, seed=9)[0]
    r0, r1 = shard.shard_bounds(rows, world, rank)
    y = oracle.gemv(synth.Q8_0, w[r0 * 28 * 34: r1 * 28 * 34], r1 - r0, COLS, x).y
    full = shard.gather_logits(torch.from_numpy(y), rows)
    out[rank] = full.numpy().tobytes()
    dist.destroy_process_group()


@pytest.mark.parametrize("rows", [2048, 2047])
def test_two_rank_full_logits_gather(rows):
    """Every rank ends with the whole logits vector, bit-identical to the
    unsharded GEMV (even and uneven shards)."""
    world = 2
    out = mp.Manager().dict()
    mp.spawn(_logits_rank, args=(world, _free_port(), rows, out), nprocs=world, join=True)
    w = synth.make_weights(synth.Q8_0, rows, COLS, seed=9)
    x = synth.make_activations(COLS, seed=9)[0]
    y = oracle.gemv(synth.Q8_0, w, rows, COLS, x).y
    for r in range(world):
        assert out[r] == y.tobytes()
