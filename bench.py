#!/usr/bin/env python3
"""Benchmark of the Q8_0 tied-embedding logits GEMV (151936 x 896, batch 1):
151936 x 896 Q8_0 weights, batch 1, fp32 logits, on 1..8 B200s (vocab-row
shards, one process per GPU).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one pass of the hot path over one activation vector: the GEMV over
this rank's vocab shard with the shard's top-1 key fused into it (one kernel
launch) and, on N > 1 GPUs, one int64 MAX all-reduce of the key (NCCL) so every
rank holds the global greedy token.  value = algorithmic bytes of all
ranks' shards (weights + x + y) / max-over-ranks device time, in GB/s.
Weights are seeded synthetic GGUF blocks (no checkpoint available); each rank
rotates over enough distinct weight copies that every step streams its shard
from HBM rather than L2 (126 MB).

--impl reference times the reference's own CPU implementation
(sim/tmac_gguf.cpp matmul_fpga_q8 + fpga_sim, compiled unmodified into
oracle/_ref/) on this host's cores for the same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

VOCAB, HIDDEN = 151936, 896
Q8_BLOCK_BYTES = 34
METRIC = json.load(open(os.path.join(ROOT, "BASELINE.json")))["metric"]
UNIT = "GB/s"
WORKLOAD = "Q8_0 tied-embedding logits GEMV 151936x896 + argmax, batch 1"
L2_BYTES = 126 * 1024 * 1024


def alg_bytes(rows, cols=HIDDEN):
    """Algorithmic bytes of one GEMV: GGUF weight blocks + fp32 x + fp32 y."""
    return rows * (cols // 32) * Q8_BLOCK_BYTES + cols * 4 + rows * 4


LAYER_BYTES = 246930432    # GGUF weight bytes of the 24 layers (12 Q8_0/Q6_K + 12 Q5_0/Q4_K mixes)
LOGITS_BYTES = 144643072   # the tied Q8_0 token_embd, 151936 x 896
MACS_PER_TOKEN = 357826560  # int16 multiply-accumulates of the 24 layers' projections per token


def decode_bytes(n_prompt, n_gen):
    """Algorithmic HBM bytes of one generate call: every forward streams the
    layer weights, every greedy step the logits weights, and attention at
    position p reads 24 layers x (k, v) x 128 floats x (p + 1)."""
    fwd = n_prompt + n_gen
    return fwd * LAYER_BYTES + n_gen * LOGITS_BYTES + 24576 * fwd * (fwd + 1) // 2


_I8_PEAK = None


def probe_i8_peak():
    """Dense int8 tensor rate of this GPU in TOPS (tmac_probe_mma_i8), best of 3."""
    global _I8_PEAK
    if _I8_PEAK is None:
        import ctypes
        import tmac_zynq_fpga_b200 as tm
        L = tm.lib()
        L.tmac_probe_mma_i8.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_double)]
        best = 0.0
        for _ in range(3):
            v = ctypes.c_double(0.0)
            tm.check(L.tmac_probe_mma_i8(0, 20000, ctypes.byref(v)))
            best = max(best, v.value)
        _I8_PEAK = best
    return _I8_PEAK


def gemm_roofline(i8_peak):
    """The prefill's largest GEMM alone: gate|up (9728 x 896 Q5_0) on 32768
    activation rows through tmac_gemm, CUDA events over 5 launches."""
    import torch
    import tmac_zynq_fpga_b200 as tm
    from tmac_zynq_fpga_b200 import synth
    rows, cols, m = 9728, 896, 32768
    w = tm.Weight(synth.Q5_0, rows, cols, synth.make_weights(synth.Q5_0, rows, cols, seed=5))
    x = torch.randn((m, cols), device="cuda")
    y = torch.empty((m, rows), device="cuda")
    for _ in range(2):
        w.gemm(x, y, m)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    cur = torch.cuda.current_stream()
    e0.record(cur)
    for _ in range(reps):
        w.gemm(x, y, m)
    e1.record(cur)
    torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / reps * 1e-3
    w.free()
    ops = 8.0 * rows * cols * m
    return {"case": "gate|up 9728x896 Q5_0, M=32768 (tmac_gemm: row quantisation + gemm_i8x4_kernel)",
            "ms": dt * 1e3, "achieved": ops / dt / 1e12, "frac": ops / dt / 1e12 / i8_peak}


def peaks():
    try:
        p = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic():
    """dram bytes per launch of the GEMV kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "q8_0_gemv_logits_151936x896.md")
    try:
        for line in open(path):
            if line.strip().startswith("dram_bytes_per_launch"):
                return float(line.split("=")[1].split()[0])
    except Exception:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons, loaded = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz, mx, pw = float(parts[1]), float(parts[2]), float(parts[3])
            except ValueError:
                continue
            smax = mx
            sm.append(mhz)
            if pw > 200:
                loaded.append(mhz)
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        use = loaded or sm
        return {"sm_mhz": statistics.median(use) if use else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm), "samples_under_load": len(loaded)}


# ------------------------------------------------------------------ reference
def _ref_worker(args):
    rows0, rows1, reps, cpus = args
    if cpus:
        os.sched_setaffinity(0, cpus)  # the caller thread and its MatmulAccel thread
    import oracle
    from tmac_zynq_fpga_b200 import synth
    rows = rows1 - rows0
    w = synth.make_weights(8, rows, HIDDEN, seed=1000 + rows0)
    x = synth.make_activations(HIDDEN, seed=0)[0]
    oracle.ref_gemv(8, w, rows, HIDDEN, x)  # warm
    t = time.perf_counter()
    for _ in range(reps):
        oracle.ref_gemv(8, w, rows, HIDDEN, x)
    return time.perf_counter() - t


def reference_throughput(rows_per_proc, procs, reps=1, pin=None):
    """The reference's matmul_fpga_q8 on `procs` host processes, each over its own
    `rows_per_proc`-row slice of the logits matrix; returns (GB/s, seconds).
    pin: per-process CPU sets (None: unpinned)."""
    import multiprocessing as mp
    ctx = mp.get_context("fork")
    with ctx.Pool(procs) as pool:
        t0 = time.perf_counter()
        times = pool.map(_ref_worker, [(i * rows_per_proc, (i + 1) * rows_per_proc, reps,
                                        None if pin is None else pin[i]) for i in range(procs)])
        wall = time.perf_counter() - t0
    elapsed = max(times)
    return procs * reps * alg_bytes(rows_per_proc) / elapsed / 1e9, elapsed, wall


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libtmac_ref.so was not built "
                          "(reference sources absent when building)"}))
        return
    cpus = sorted(os.sched_getaffinity(0))
    cores = len(cpus)
    # each process runs two busy threads (the caller and fpga_sim's MatmulAccel
    # FSM thread, sim/fpga_sim.hpp:195-205): one process per two cores, pinned
    procs = max(1, cores // 2)
    pin = [set(cpus[2 * i:2 * i + 2]) for i in range(procs)]
    rows_per_proc = 4096  # ~50 ms of reference work per process per step
    vals = []
    for _ in range(min(args.warmup, 3)):
        reference_throughput(rows_per_proc, procs, pin=pin)
    steps = min(args.steps, 50)
    t0 = time.perf_counter()
    for _ in range(steps):
        vals.append(reference_throughput(rows_per_proc, procs, pin=pin)[0])
    total = time.perf_counter() - t0
    v = statistics.median(vals)
    sample = (f"{procs} processes (2 cores each: caller + fpga_sim MatmulAccel thread) x {rows_per_proc} rows "
              f"of the 151936x896 Q8_0 logits matrix per step, median of {steps} steps (matmul_fpga_q8)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / max(args.steps, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int16/int64",
        "data": "synthetic", "config": {"workload": WORKLOAD, "parallelism": f"{procs} host processes"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": 2 * procs, "kind": "reference", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "decode": reference_decode_sample(),
    }))


def reference_decode_sample():
    """The reference engine's own decode (process_prompt + greedy steps of
    sim/tmac_gguf.cpp, all four --fpga-* switches, oracle/_ref) on the same
    seed-0 synthetic model: a 1-token prompt and 2 greedy steps, i.e. 3 forwards
    and 2 logits GEMVs, on one process pinned to two cores.  Sampled: the full
    8 + 64 run takes minutes of host time."""
    import ctypes
    import multiprocessing as mp
    ctx = mp.get_context("fork")
    with ctx.Pool(1) as pool:
        return pool.apply(_ref_decode_worker)


def _ref_decode_worker():
    import ctypes
    import oracle
    from tmac_zynq_fpga_b200 import model
    cpus = sorted(os.sched_getaffinity(0))[:2]
    os.sched_setaffinity(0, set(cpus))
    path = model.default_model_path(0)
    R = oracle.ref()
    R.ref_decode.restype = ctypes.c_int
    R.ref_decode.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                             ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    prompt = model.prompt_tokens(8, seed=0)[:1].copy()
    n_gen = 2
    toks = np.zeros(n_gen, np.int32)
    t0 = time.perf_counter()
    n = R.ref_decode(path.encode(), prompt.ctypes.data, len(prompt), n_gen, 1, toks.ctypes.data, None, None)
    dt = time.perf_counter() - t0
    fwd = len(prompt) + n_gen
    return {"tok_s": n_gen / dt, "ms_per_forward": 1000 * dt / fwd, "seconds": dt, "prompt_tokens": len(prompt),
            "generated": int(n), "cores": len(cpus), "sampled": True,
            "config": "reference engine (tmac_gguf.cpp process_prompt + greedy steps, all --fpga-* switches) "
                      "on the seed-0 synthetic Qwen2-0.5B-shaped model; includes load_tmac of the model file"}


# ------------------------------------------------------------------- ours
def cpu_baseline_single():
    """The reference (oracle/_ref) on one host process pinned to two cores (its
    caller thread and fpga_sim's MatmulAccel thread): the median of 5 runs, each
    4 calls of matmul_fpga_q8 over a quarter of the logits matrix (~10 s)."""
    import oracle
    if not oracle.ref_available():
        return None
    rows = 37984  # a quarter of the vocabulary: ~0.45 s per call
    pin = [set(sorted(os.sched_getaffinity(0))[:2])]
    runs = [reference_throughput(rows, 1, reps=4, pin=pin)[0] for _ in range(5)]
    return {"value": statistics.median(runs), "unit": UNIT, "cores": 2, "kind": "reference",
            "sample": f"median of 5 runs of 4 x matmul_fpga_q8 over a {rows}x896 slice of the logits matrix, "
                      f"1 process pinned to 2 cores (caller + fpga_sim MatmulAccel FSM thread); "
                      f"runs {', '.join(f'{r:.4f}' for r in runs)} GB/s"}


def model_extras(world=1, rank=0):
    """Full decode and batched prefill through the public model API: greedy decode
    (8-token prompt + 64 steps, tokens checked against the reference's committed
    fixture; one GPU only: decode does not shard) and batched prefill of 64 x 512
    tokens, sharded by sequence over the ranks (no collective on the data path;
    time = max over ranks).  Wall clock per call (host buffers in and out), after
    a warm-up call."""
    import torch
    import torch.distributed as dist
    import tmac_zynq_fpga_b200 as tm
    from tmac_zynq_fpga_b200 import model, shard
    g = np.load(os.path.join(ROOT, "tests", "golden", "decode_greedy_seed0.npz"))
    m = tm.Model(model.default_model_path(int(g["model_seed"])), switches=tm.SW_ALL, max_seq=512,
                 device=torch.cuda.current_device())
    decode = None
    if world == 1:
        prompt, ref = g["prompt"].astype(np.int32), g["tokens"]
        n = len(ref)
        toks, _ = m.generate(prompt, n)
        reps = 5
        t0 = time.perf_counter()
        for _ in range(reps):
            toks, _ = m.generate(prompt, n)
        dt = (time.perf_counter() - t0) / reps
        fwd = len(prompt) + n
        dbytes = decode_bytes(len(prompt), n)
        pk, pk_kind = peaks()
        decode = {"tok_s": n / dt, "ms_per_call": 1000 * dt, "prompt_tokens": len(prompt), "generated": n,
                  "ms_per_forward": 1000 * dt / fwd,
                  "roofline": {"bound": "hbm", "achieved": dbytes / dt / 1e9, "peak": pk, "unit": "GB/s",
                               "frac": dbytes / dt / 1e9 / pk, "peak_kind": f"{pk_kind} hbm_gbs (copy)",
                               "bytes_per_call": dbytes,
                               "bytes": f"{fwd} forwards x {LAYER_BYTES} B of layer weights + {n} x "
                                        f"{LOGITS_BYTES} B of logits weights + KV reads 24576 B x (pos + 1)"},
                  "tokens_match_reference": bool(np.array_equal(toks, ref)),
                  "engine": {1: "persistent kernel (one cooperative launch per token) + logits GEMV",
                             0: "per-kernel engine (CUDA graphs)"}.get(m.decode_engine(), "unknown"),
                  "config": "Qwen2-0.5B-shaped decode: 24 layers, mixed Q5_0/Q8_0/Q4_K/Q6_K, 512-slot KV, "
                            "greedy",
                  "api": "tmac_model_generate"}
    rng = np.random.default_rng(0)
    ptoks = rng.integers(0, VOCAB, size=(64, 512)).astype(np.int32)
    s0, s1 = shard.sequence_shard(len(ptoks), world, rank)
    mine = ptoks[s0:s1]
    nxt, _ = m.prefill(mine)
    reps = 3
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(reps):
        nxt2, _ = m.prefill(mine)
    dt = torch.tensor([(time.perf_counter() - t0) / reps], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(dt, op=dist.ReduceOp.MAX)
        allnxt = shard.gather_next_tokens(nxt2, len(ptoks))
    else:
        allnxt = nxt2
    dt = float(dt.item())
    i8_ops = 8 * MACS_PER_TOKEN * ptoks.size  # Mode E: 4 int8 MMAs of 2 ops per int16 multiply-accumulate
    i8_peak = probe_i8_peak() if rank == 0 else None
    prefill = {"tok_s": ptoks.size / dt, "ms_per_call": 1000 * dt, "n_seq": len(ptoks), "len": ptoks.shape[1],
               "roofline": None if not i8_peak else {
                   "bound": "tensor", "achieved": i8_ops / dt / 1e12, "peak": i8_peak, "unit": "TOPS (int8)",
                   "frac": i8_ops / dt / 1e12 / (i8_peak * world),
                   "peak_kind": "measured on this GPU: tcgen05.mma kind::i8 M128 N256 back to back "
                                "(tmac_probe_mma_i8)",
                   "ops": f"8 x {MACS_PER_TOKEN} int8 ops per token (4 MMAs per int16 MAC) over all projections; "
                          "the whole call (attention, norms, logits included) is timed",
                   "gemm_only": gemm_roofline(i8_peak)},
               "n_gpus": world, "seq_per_gpu": s1 - s0, "scaling": "strong (fixed 64 x 512 batch)",
               "deterministic": bool(np.array_equal(nxt, nxt2)), "next_tokens_gathered": int(len(allnxt)),
               "config": "batched prefill of the same model: 64 x 512 tokens, sequence shards, exact "
                         "int16 x int16 on tcgen05 int8 MMAs",
               "api": "tmac_model_prefill"}
    m.free()
    return decode, prefill


def gemv_shapes():
    """The other GEMV configurations (configs 1 and 3): device time per GEMV in a
    CUDA graph of back-to-back launches with programmatic dependent launch,
    over rotating weight copies larger than L2 (so every launch streams its
    weights from HBM), fp32 x in / fp32 y out.  At these sizes (0.5-3.6 MB of
    weights) a launch's fixed latency, not HBM bandwidth, bounds the time."""
    import torch
    import tmac_zynq_fpga_b200 as tm
    from tmac_zynq_fpga_b200 import synth
    pk, _ = peaks()
    out = []
    cases = [("attn_q Q5_0", synth.Q5_0, 896, 896, 1),
             ("ffn_down Q4_K", synth.Q4_K, 896, 4864, 1),
             ("ffn_down Q6_K", synth.Q6_K, 896, 4864, 1),
             ("ffn_down Q4_K", synth.Q4_K, 896, 4864, 16),
             ("ffn_down Q6_K", synth.Q6_K, 896, 4864, 16),
             ("ffn_gate Q5_0", synth.Q5_0, 4864, 896, 1),
             ("ffn_gate|up Q5_0", synth.Q5_0, 9728, 896, 1)]
    L = tm.lib()
    for name, qt, rows, cols, batch in cases:
        raw = synth.make_weights(qt, rows, cols, seed=1)
        w0 = tm.Weight(qt, rows, cols, raw)
        ncopy = max(2, int(2 * L2_BYTES // w0.device_bytes()) + 1)
        ws = [w0] + [tm.Weight(qt, rows, cols, raw) for _ in range(ncopy - 1)]
        x = torch.from_numpy(synth.make_activations(cols, batch=batch, seed=1)).cuda()
        y = torch.empty((batch, rows), device="cuda")
        L.tmac_reserve(0, batch, cols)
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            for w in ws:
                w.gemv(x, y, batch=batch, stream=st)
        torch.cuda.synchronize()
        prev = L.tmac_set_pdl(1)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for w in ws:
                w.gemv(x, y, batch=batch, stream=st)
        L.tmac_set_pdl(prev)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        cur = torch.cuda.current_stream()  # replay() runs on the current stream
        e0.record(cur)
        for _ in range(reps):
            g.replay()
        e1.record(cur)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / (reps * len(ws)) * 1e3
        blk = {synth.Q5_0: 22 / 32, synth.Q4_K: 144 / 256, synth.Q6_K: 210 / 256}[qt]
        alg = rows * cols * blk + batch * (rows + cols) * 4
        out.append({"case": name, "rows": rows, "cols": cols, "batch": batch, "us_per_gemv": us,
                    "gbs": alg / us / 1e3, "frac_of_hbm": alg / us / 1e3 / pk})
        for w in ws:
            w.free()
    out.append(hw_chain_shape(pk))
    assert tm.device_error(0) == 0
    return out


def hw_chain_shape(pk):
    """attn_q 896x896 Q5_0 through the FPGA's own descriptor format: one chain of
    D hardware descriptors (type 1, num_tiles = 224 4-row tiles each), every one
    over its own copy of the matrix so that the chain streams more than twice
    L2 from HBM; one tmac_chain_run_hw call per chain, CUDA events around it.
    Per descriptor: int16 x (from the arena) in, 896 int64 rows out."""
    import torch
    from tmac_zynq_fpga_b200 import hwchain, synth
    rows = cols = 896
    w = synth.make_weights(synth.Q5_0, rows, cols, seed=1)
    xq = np.clip(np.round(synth.make_activations(cols, seed=1)[0] * 8000), -32768, 32767).astype(np.int16)
    tiles = hwchain.pack_q5_0_tiles(w, rows).reshape(-1)
    D = int(2 * L2_BYTES // tiles.nbytes) + 1
    base = 0x10000000
    act = base + 32 * D
    wt0 = (act + 2 * cols + 255) // 256 * 256
    stride = (tiles.nbytes + 255) // 256 * 256
    res0 = wt0 + D * stride
    arena = np.zeros(res0 - base + D * rows * 8, np.uint8)
    for i in range(D):
        nxt = base + 32 * (i + 1) if i + 1 < D else 0
        arena[32 * i:32 * i + 32] = np.frombuffer(
            hwchain.desc_bytes(nxt, wt0 + i * stride, act, res0 + i * rows * 8, hwchain.Q5_0, 0, rows // 4,
                               2 * cols), np.uint8)
        arena[wt0 - base + i * stride:wt0 - base + i * stride + tiles.nbytes] = tiles
    arena[act - base:act - base + 2 * cols] = xq.view(np.uint8)
    dev = torch.from_numpy(arena).cuda()
    for _ in range(2):
        hwchain.chain_run_hw(dev, arena.nbytes, base, base, arena_host=arena)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    cur = torch.cuda.current_stream()
    e0.record(cur)
    for _ in range(reps):
        hwchain.chain_run_hw(dev, arena.nbytes, base, base, arena_host=arena, stream=cur)
    e1.record(cur)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / (reps * D) * 1e3
    alg = rows * cols * 22 // 32 + cols * 2 + rows * 8
    return {"case": "attn_q Q5_0 as one hardware descriptor (num_tiles=224) per matrix, tmac_chain_run_hw",
            "rows": rows, "cols": cols, "batch": 1, "descriptors_per_chain": D, "us_per_gemv": us,
            "gbs": alg / us / 1e3, "frac_of_hbm": alg / us / 1e3 / pk}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-model", action="store_true", help="skip the decode / prefill measurements")
    ap.add_argument("--no-graph", action="store_true",
                    help="issue the timed steps one by one from Python instead of replaying a CUDA graph of them")
    ap.add_argument("--no-pdl", action="store_true",
                    help="launch each step's kernel after the previous one ends (no programmatic dependent launch)")
    ap.add_argument("--top1-only", dest="full_logits", action="store_false",
                    help="N > 1: only the global greedy token on every rank, not the whole logits vector")
    ap.add_argument("--full-logits", dest="full_logits", action="store_true", default=True,
                    help="(default) N > 1: every rank also ends each step with the whole logits vector, as "
                         "get_logits_q8 returns it: stored over NVLink by the GEMV itself with the fused "
                         "exchange, else an NCCL all-gather")
    ap.add_argument("--collective", choices=["fused", "peer", "nccl"], default="fused",
                    help="top-1 merge across ranks: inside the logits GEMV over NVLink peer memory, "
                         "a separate peer-memory exchange kernel, or an NCCL all-reduce")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist
    import tmac_zynq_fpga_b200 as tm
    from tmac_zynq_fpga_b200 import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))

    # vocab-row shard of this rank
    r0, r1 = rank * VOCAB // world, (rank + 1) * VOCAB // world
    rows = r1 - r0
    raw = synth.make_weights(8, VOCAB, HIDDEN, seed=0)
    shard = raw[r0 * (HIDDEN // 32) * Q8_BLOCK_BYTES: r1 * (HIDDEN // 32) * Q8_BLOCK_BYTES]
    shard_dev = torch.from_numpy(shard).cuda()
    w0 = tm.Weight(8, rows, HIDDEN, shard_dev, device=local)
    del shard_dev
    per_copy = w0.device_bytes()
    ncopies = max(2, -(-2 * L2_BYTES // per_copy))
    weights = [w0]
    for _ in range(ncopies - 1):
        weights.append(tm.Weight(8, rows, HIDDEN, torch.from_numpy(shard).cuda(), device=local))
    torch.cuda.synchronize()
    x = torch.from_numpy(synth.make_activations(HIDDEN, seed=0)).cuda()
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream()

    # top-1 merge across ranks over NVLink peer memory (fused into the logits
    # GEMV, or a kernel of its own), checked first against the NCCL all-reduce
    # of the shard keys; NCCL all-reduce if that check fails
    merge, merge_kind, fused = None, "none", False
    if world > 1:
        merge_kind = "nccl int64 MAX all-reduce"
        if args.collective in ("fused", "peer"):
            from tmac_zynq_fpga_b200 import shard
            try:
                # --full-logits with the fused exchange: the GEMV also stores its rows
                # into every rank's full-logits vector over NVLink (no NCCL all-gather)
                xchg = shard.PeerTop1(local, vocab=VOCAB if (args.full_logits and args.collective == "fused") else 0)
                weights[0].gemv_top1(x, y, key, index_base=r0, stream=stream)
                ref = key.clone()
                dist.all_reduce(ref, op=dist.ReduceOp.MAX)
                if args.collective == "fused":
                    xchg.gemv_top1(weights[0], x, y, key, r0, stream)
                else:
                    xchg(key, stream)
                torch.cuda.synchronize()
                if not torch.equal(ref, key) or tm.device_error(local) != 0:
                    raise RuntimeError("peer exchange disagrees with the NCCL all-reduce")
                merge = xchg
                fused = args.collective == "fused"
                merge_kind = ("top-1 exchange over NVLink peer memory inside the GEMV's last CTA "
                              "(tmac_xchg_gemv_top1)" if fused else
                              "NVLink peer-memory exchange kernel (tmac_xchg_top1)")
            except Exception as e:  # keep NCCL
                merge_kind = f"nccl int64 MAX all-reduce (peer exchange unavailable: {e})"

    peer_full = fused and merge is not None and merge.vocab > 0
    gather = world > 1 and args.full_logits and not peer_full
    y_full = torch.empty(VOCAB, dtype=torch.float32, device="cuda") if gather else None

    def step(i, st=None):
        # logits of this rank's vocab shard + their top-1 key, then the global
        # greedy token on every rank (and, with --full-logits, the whole vector)
        st = stream if st is None else st
        w = weights[i % ncopies]
        if fused:
            merge.gemv_top1(w, x, y, key, r0, st)
        else:
            w.gemv_top1(x, y, key, index_base=r0, stream=st)
            if world > 1:
                if merge is not None:
                    merge(key, stream)
                else:
                    dist.all_reduce(key, op=dist.ReduceOp.MAX)
        if gather:
            from tmac_zynq_fpga_b200 import shard as _shard
            _shard.gather_logits(y, VOCAB, out=y_full)

    # consecutive steps' kernels: the next one's prologue and weight copies may
    # start while the previous one finishes (tmac_set_pdl; results unchanged)
    prev_pdl = tm.lib().tmac_set_pdl(0 if args.no_pdl else 1)
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if tm.device_error(local) != 0:
        raise SystemExit("a kernel recorded a device-side error during warm-up")
    # The timed steps run as replays of a CUDA graph of G consecutive steps (one
    # kernel launch each, programmatic dependent launch between them) when a
    # step is a single launch: at N > 1 a shard's GEMV takes a few microseconds,
    # less than issuing it from Python.  G is even (the exchange alternates
    # buffer halves by step parity) and divides K, so exactly K steps are timed.
    graph, G = None, 0
    if not args.no_graph and (world == 1 or (fused and not gather)):
        G = next((g for g in range(64, 1, -1) if g % 2 == 0 and args.steps % g == 0), 0)
        if G:
            cap = torch.cuda.Stream()
            cap.wait_stream(stream)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=cap):
                for i in range(G):
                    step(i, cap)
            torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    if graph is not None:
        for _ in range(args.steps // G):
            graph.replay()  # on the current stream
    else:
        for i in range(args.steps):
            step(i)
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    total_bytes = alg_bytes(VOCAB) + (world - 1) * HIDDEN * 4  # every rank reads x
    value = total_bytes / (ms_per_step * 1e-3) / 1e9
    kernel_us = ms / args.steps * 1e3  # one launch per step on this rank
    tm.lib().tmac_set_pdl(prev_pdl)

    # At N > 1: this rank's shard GEMV alone (fused top-1 key, no exchange), timed
    # the same way, so the line shows what the exchange adds to the step.
    shard_alone = None
    if world > 1:
        la_us, la_failed, la_note = 0.0, 0.0, ""
        la_pdl = tm.lib().tmac_set_pdl(0 if args.no_pdl else 1)  # as in the timed steps
        try:
            key_l = torch.zeros(1, dtype=torch.int64, device="cuda")
            cap_l = torch.cuda.Stream()
            cap_l.wait_stream(stream)
            with torch.cuda.stream(cap_l):
                for i in range(args.warmup):
                    weights[i % ncopies].gemv_top1(x, y, key_l, index_base=r0, stream=cap_l)
            torch.cuda.synchronize()
            g_l = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_l, stream=cap_l):
                for i in range(50):
                    weights[i % ncopies].gemv_top1(x, y, key_l, index_base=r0, stream=cap_l)
            torch.cuda.synchronize()
            g_l.replay()
            torch.cuda.synchronize()
            l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            l0.record(stream)
            for _ in range(20):
                g_l.replay()
            l1.record(stream)
            torch.cuda.synchronize()
            la_us = l0.elapsed_time(l1) / 1000 * 1e3
        except Exception as ex:  # reported, never fatal: the step above is the measurement
            la_failed, la_note = 1.0, str(ex)[:200]
        tm.lib().tmac_set_pdl(la_pdl)
        la = torch.tensor([la_us, la_failed], dtype=torch.float64, device="cuda")
        dist.all_reduce(la, op=dist.ReduceOp.MAX)
        shard_alone = ({"error": la_note or "failed on another rank"} if la[1].item() > 0 else
                       {"us_per_step": float(la[0].item()), "steps": 1000,
                        "what": "this rank's shard GEMV with its top-1 key, no exchange (CUDA graph of 50, "
                                "max over ranks); the step minus this is the exchange's cost"})

    # e2e: the public host-buffer entry (tmac_gemv_host): H2D x, GEMV, D2H y per step.
    xh = torch.from_numpy(synth.make_activations(HIDDEN, seed=0)).pin_memory()
    yh = torch.empty(rows, dtype=torch.float32).pin_memory()
    L = tm.lib()
    e2e_steps = max(10, args.steps // 10)
    for i in range(args.warmup):
        tm.check(L.tmac_gemv_host(weights[i % ncopies].handle, xh.data_ptr(), yh.data_ptr(), 1))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    d0 = torch.cuda.Event(enable_timing=True)
    d1 = torch.cuda.Event(enable_timing=True)
    d0.record(torch.cuda.default_stream())
    for i in range(e2e_steps):
        tm.check(L.tmac_gemv_host(weights[i % ncopies].handle, xh.data_ptr(), yh.data_ptr(), 1))
    d1.record(torch.cuda.default_stream())
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([d0.elapsed_time(d1) / e2e_steps], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    clocks = sampler.stop()
    e2e_val = total_bytes / (float(e2e_ms.item()) * 1e-3) / 1e9
    assert tm.device_error(local) == 0
    # the greedy token of the last step must be the global argmax of the logits
    tok = tm.top1_decode(key.item())[1]
    yl = y.cpu().numpy()
    if world == 1:
        assert tok == int(np.argmax(yl)), "fused top-1 disagrees with argmax of the logits"

    decode = prefill = None
    if not args.no_model:
        decode, prefill = model_extras(world, rank)
    shapes = gemv_shapes() if (world == 1 and not args.no_model) else None

    if rank == 0:
        pk, pk_kind = peaks()
        achieved = alg_bytes(rows) / (kernel_us * 1e-6) / 1e9
        traffic = profile_traffic()
        if traffic is not None and world > 1:
            traffic = traffic * rows / VOCAB
        cpu = None if (args.no_cpu_baseline or world > 1) else cpu_baseline_single()
        out = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int16/int64", "data": "synthetic",
            "config": {"workload": WORKLOAD, "rows": VOCAB, "cols": HIDDEN, "batch": 1,
                       "step": "shard logits GEMV with fused top-1 key" + (f" + {merge_kind}" if world > 1 else "")
                               + (" + NCCL all-gather of the logits shards" if gather else "")
                               + (" + full logits stored into every rank over NVLink inside the GEMV"
                                  if peer_full else ""),
                       "greedy_token": tok,
                       "parallelism": f"vocab-row shards x{world}", "shard_rows": rows,
                       "launch": ("back-to-back, no programmatic dependent launch" if args.no_pdl else
                                  "programmatic dependent launch between steps (tmac_set_pdl)")
                                 + (f"; CUDA graph of {G} steps replayed {args.steps // G} times" if graph is not None
                                    else "; steps issued one by one"),
                       "l2": f"inputs larger than L2: {ncopies} rotating weight copies of "
                             f"{per_copy / 1e6:.1f} MB per rank"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk, "unit": "GB/s",
                         "frac": achieved / pk, "peak_kind": f"{pk_kind} hbm_gbs (copy)",
                         "kernel": "q8_gemv_kernel", "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": HIDDEN * 4,
                    "d2h_bytes_per_step": rows * 4, "api": "tmac_gemv_host", "steps": e2e_steps},
            "gpu_launches": args.steps * (2 if (merge is not None and not fused) else 1),
            "clocks": clocks,
            "shard_alone": shard_alone,
            "decode": decode,
            "gemv_shapes": shapes,
            "prefill": prefill,
        }
        print(json.dumps(out))
    for w in weights:
        w.free()
    if merge is not None:
        merge.free()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
