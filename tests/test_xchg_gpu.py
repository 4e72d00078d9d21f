"""Top-1 merge of vocab-sharded logits over peer memory (tmac_xchg_*).

The global greedy token over every rank's shard must be the argmax of the whole
logits vector (sim/tmac_gguf.cpp:1974-1990 samples from one full vector).  The
fused form (tmac_xchg_gemv_top1: the exchange inside the Q8_0 GEMV's last CTA)
must give the same y and key as tmac_gemv_top1 followed by tmac_xchg_top1,
step after step, with no key reset between steps.  One rank exercises the
publish / acquire / step protocol on one GPU; two ranks (two GPUs, one process
each) the peer stores."""
import ctypes
import os
import socket

import numpy as np
import pytest

import tmac_zynq_fpga_b200 as tm
from tmac_zynq_fpga_b200 import synth

pytestmark = pytest.mark.gpu

Q8_BLOCK_BYTES = 34


def _xchg_world1(device=0):
    L = tm.lib()
    h = ctypes.c_void_p()
    tm.check(L.tmac_xchg_create(device, 1, 0, ctypes.byref(h)))
    buf = (ctypes.c_uint8 * 64)()
    tm.check(L.tmac_xchg_ipc_handle(h, buf))
    tm.check(L.tmac_xchg_open(h, bytes(buf)))
    return h


@pytest.mark.parametrize("qtype,rows,cols", [(synth.Q8_0, 5000, 896), (synth.Q8_0, 151936, 896),
                                             (synth.Q5_0, 4864, 896)])
def test_fused_exchange_one_rank_matches_gemv_top1(qtype, rows, cols):
    torch = pytest.importorskip("torch")
    L = tm.lib()
    w = tm.Weight(qtype, rows, cols, synth.make_weights(qtype, rows, cols, seed=31))
    h = _xchg_world1()
    try:
        base = 1000
        for step in range(6):
            x = torch.from_numpy(synth.make_activations(cols, seed=40 + step) * (1 + step)).cuda()
            y_ref = torch.empty(rows, device="cuda")
            k_ref = torch.zeros(1, dtype=torch.int64, device="cuda")
            w.gemv_top1(x, y_ref, k_ref, index_base=base)
            y = torch.full((rows,), float("nan"), device="cuda")
            key = torch.full((1,), -1, dtype=torch.int64, device="cuda")  # never reset by the caller
            if step % 3 == 2:  # mix in the separate exchange kernel: the step count is shared
                w.gemv_top1(x, y, key, index_base=base)
                tm.check(L.tmac_xchg_top1(h, key.data_ptr(), None))
            else:
                tm.check(L.tmac_xchg_gemv_top1(h, w.handle, x.data_ptr(), y.data_ptr(), key.data_ptr(), base, None))
            torch.cuda.synchronize()
            assert tm.device_error(0) == 0
            assert torch.equal(y, y_ref)
            assert key.item() == k_ref.item()
            assert tm.top1_decode(key.item())[1] == base + int(np.argmax(y_ref.cpu().numpy()))
    finally:
        L.tmac_xchg_free(h)


@pytest.mark.parametrize("fused", [True, False])
def test_exchange_wait_runs_out_when_a_rank_never_publishes(fused):
    """Rank 1 of a two-rank exchange is a second buffer in this process that no
    kernel ever writes (a flag nothing sets).  With a 50 ms wait limit, rank 0's
    wait gives up: the call returns, tmac_device_error reports TMAC_ERR_TIMEOUT,
    the caller's key is left as it was, and the device still runs a normal GEMV
    correctly afterwards (the counterpart of MatmulAccel::wait_done's timeout,
    sim/fpga_sim.hpp:232-241)."""
    torch = pytest.importorskip("torch")
    import time
    L = tm.lib()
    L.tmac_set_wait_limit_ns.argtypes = [ctypes.c_int, ctypes.c_uint64]
    rows, cols = 2048, 896
    w = tm.Weight(synth.Q8_0, rows, cols, synth.make_weights(synth.Q8_0, rows, cols, seed=33))
    h0, h1 = ctypes.c_void_p(), ctypes.c_void_p()
    tm.check(L.tmac_xchg_create(0, 2, 0, ctypes.byref(h0)))
    tm.check(L.tmac_xchg_create(0, 2, 1, ctypes.byref(h1)))
    try:
        handles = (ctypes.c_uint8 * 128)()
        tm.check(L.tmac_xchg_ipc_handle(h0, ctypes.byref(handles, 0)))
        tm.check(L.tmac_xchg_ipc_handle(h1, ctypes.byref(handles, 64)))
        tm.check(L.tmac_xchg_open(h0, bytes(handles)))
        assert tm.device_error(0) == 0
        tm.check(L.tmac_set_wait_limit_ns(0, 50_000_000))
        x = torch.from_numpy(synth.make_activations(cols, seed=34)).cuda()
        y = torch.empty(rows, device="cuda")
        sentinel = 0x1234567
        key = torch.full((1,), sentinel, dtype=torch.int64, device="cuda")
        t0 = time.time()
        if fused:
            tm.check(L.tmac_xchg_gemv_top1(h0, w.handle, x.data_ptr(), y.data_ptr(), key.data_ptr(), 0, None))
        else:
            w.gemv_top1(x, y, key)
            key.fill_(sentinel)
            tm.check(L.tmac_xchg_top1(h0, key.data_ptr(), None))
        torch.cuda.synchronize()
        assert time.time() - t0 < 10.0
        assert tm.device_error(0) == -7          # TMAC_ERR_TIMEOUT
        assert key.item() == sentinel            # the key is left as it was
        assert tm.device_error(0) == 0           # read-and-clear
    finally:
        L.tmac_set_wait_limit_ns(0, 2_000_000_000)
        L.tmac_xchg_free(h0)
        L.tmac_xchg_free(h1)
    # the context is still usable: a plain GEMV + top-1 is right
    y2 = torch.empty(rows, device="cuda")
    k2 = torch.zeros(1, dtype=torch.int64, device="cuda")
    w.gemv_top1(x, y2, k2)
    torch.cuda.synchronize()
    assert tm.device_error(0) == 0
    assert tm.top1_decode(k2.item())[1] == int(np.argmax(y2.cpu().numpy()))
    w.free()


def test_fused_exchange_rejects_bad_arguments():
    torch = pytest.importorskip("torch")
    L = tm.lib()
    w = tm.Weight(synth.Q8_0, 256, 896, synth.make_weights(synth.Q8_0, 256, 896, seed=3))
    h = ctypes.c_void_p()
    tm.check(L.tmac_xchg_create(0, 2, 0, ctypes.byref(h)))
    try:
        x = torch.zeros(896, device="cuda")
        y = torch.zeros(256, device="cuda")
        key = torch.zeros(1, dtype=torch.int64, device="cuda")
        # rank 1 not mapped yet: refused before any launch (nothing waits)
        assert L.tmac_xchg_gemv_top1(h, w.handle, x.data_ptr(), y.data_ptr(), key.data_ptr(), 0, None) != 0
        assert L.tmac_xchg_gemv_top1(h, w.handle, None, y.data_ptr(), key.data_ptr(), 0, None) != 0
    finally:
        L.tmac_xchg_free(h)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, rows, cols, fused, out, full=False):
    import torch
    import torch.distributed as dist
    from tmac_zynq_fpga_b200 import shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        raw = synth.make_weights(synth.Q8_0, rows, cols, seed=77)
        r0, r1 = rank * rows // world, (rank + 1) * rows // world
        blk = (cols // 32) * Q8_BLOCK_BYTES
        w = tm.Weight(synth.Q8_0, r1 - r0, cols, raw[r0 * blk:r1 * blk], device=rank)
        xchg = shard.PeerTop1(rank, vocab=rows if full else 0)
        keys, fulls = [], []
        for step in range(8):
            x = torch.from_numpy(synth.make_activations(cols, seed=50 + step) * (1 + step)).cuda()
            y = torch.empty(r1 - r0, device="cuda")
            key = torch.zeros(1, dtype=torch.int64, device="cuda")
            if fused:
                xchg.gemv_top1(w, x, y, key, r0)
            else:
                w.gemv_top1(x, y, key, index_base=r0)
                xchg(key)
            torch.cuda.synchronize()
            keys.append(key.item())
            if full:
                fulls.append(xchg.logits().cpu().numpy().copy())
        assert tm.device_error(rank) == 0
        out.put((rank, (keys, fulls) if full else keys))
        dist.barrier()
        xchg.free()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fused", [True, False])
def test_two_ranks_merge_to_global_argmax(fused):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    rows, cols = 20000, 896
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, rows, cols, fused, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            r, keys = q.get(timeout=300)
            got[r] = keys
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    w = tm.Weight(synth.Q8_0, rows, cols, synth.make_weights(synth.Q8_0, rows, cols, seed=77))
    for step in range(8):
        x = torch.from_numpy(synth.make_activations(cols, seed=50 + step) * (1 + step)).cuda()
        y = torch.empty(rows, device="cuda")
        key = torch.zeros(1, dtype=torch.int64, device="cuda")
        w.gemv_top1(x, y, key)
        assert got[0][step] == got[1][step] == key.item(), step


def test_two_ranks_full_logits_over_peer_memory():
    """The fused exchange with the full logits (tmac_xchg_create_logits): each
    rank's shard GEMV also stores its rows into both ranks' full vectors over
    NVLink, so after every step both ranks hold the whole logits vector, bit
    for bit the unsharded GEMV's, and the same greedy key."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    rows, cols = 20000, 896
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, rows, cols, True, q, True)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            r, res = q.get(timeout=300)
            got[r] = res
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    w = tm.Weight(synth.Q8_0, rows, cols, synth.make_weights(synth.Q8_0, rows, cols, seed=77))
    for step in range(8):
        x = torch.from_numpy(synth.make_activations(cols, seed=50 + step) * (1 + step)).cuda()
        y = torch.empty(rows, device="cuda")
        key = torch.zeros(1, dtype=torch.int64, device="cuda")
        w.gemv_top1(x, y, key)
        yh = y.cpu().numpy()
        for r in range(2):
            keys, fulls = got[r]
            assert keys[step] == key.item(), step
            np.testing.assert_array_equal(fulls[step].view(np.int32), yh.view(np.int32), err_msg=f"rank {r} step {step}")


def test_one_rank_full_logits_buffer():
    """World 1: the full-logits buffer of each step equals y (both parities)."""
    torch = pytest.importorskip("torch")
    from tmac_zynq_fpga_b200 import shard
    L = tm.lib()
    rows, cols = 3000, 896
    w = tm.Weight(synth.Q8_0, rows, cols, synth.make_weights(synth.Q8_0, rows, cols, seed=41))
    h = ctypes.c_void_p()
    L.tmac_xchg_create_logits.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64,
                                          ctypes.POINTER(ctypes.c_void_p)]
    tm.check(L.tmac_xchg_create_logits(0, 1, 0, rows, ctypes.byref(h)))
    try:
        buf = (ctypes.c_uint8 * 64)()
        tm.check(L.tmac_xchg_ipc_handle(h, buf))
        tm.check(L.tmac_xchg_open(h, bytes(buf)))
        p = ctypes.c_void_p()
        L.tmac_xchg_logits.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        assert L.tmac_xchg_logits(h, ctypes.byref(p)) != 0  # no step yet
        for step in range(3):
            x = torch.from_numpy(synth.make_activations(cols, seed=60 + step)).cuda()
            y = torch.empty(rows, device="cuda")
            key = torch.zeros(1, dtype=torch.int64, device="cuda")
            tm.check(L.tmac_xchg_gemv_top1(h, w.handle, x.data_ptr(), y.data_ptr(), key.data_ptr(), 0, None))
            tm.check(L.tmac_xchg_logits(h, ctypes.byref(p)))
            full = shard.device_view(p.value, rows).cpu().numpy()
            np.testing.assert_array_equal(full.view(np.int32), y.cpu().numpy().view(np.int32))
        assert tm.device_error(0) == 0
    finally:
        L.tmac_xchg_free(h)
        w.free()
