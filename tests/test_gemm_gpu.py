"""Tensor-core batched matmul (tmac_gemm, prefill) against the GEMV.

tmac_gemm runs every activation row through the same arithmetic as one
tmac_gemv call (the reference's matmul_fpga_* per token), on tcgen05 int8 MMAs
over byte planes of the exact int16 weights.  Bar: y and the int64 row sums
identical to tmac_gemv with batch m, bit for bit, including partial tiles
(m and rows not multiples of 128) and K not a multiple of the 128-byte stage.
"""
import numpy as np
import pytest


def per_row_gemv(w, x, m, rows):
    """The reference for tmac_gemm: one batch-1 CUDA-core GEMV per activation
    row (tmac_gemv itself sends batches of 8..64 to the tensor cores)."""
    import torch
    y = torch.empty((m, rows), device="cuda")
    acc = torch.zeros((m, rows), dtype=torch.int64, device="cuda")
    for i in range(m):
        w.gemv(x[i], y[i], batch=1, row_acc=acc[i])
    return y, acc

import tmac_zynq_fpga_b200 as tm
from tmac_zynq_fpga_b200 import synth

pytestmark = pytest.mark.gpu

CASES = [(synth.Q5_0, 1152, 896, 300), (synth.Q5_0, 200, 96, 129), (synth.Q4_K, 896, 4864, 200),
         (synth.Q6_K, 896, 4864, 131), (synth.Q6_K, 136, 768, 64)]


@pytest.mark.parametrize("qtype,rows,cols,m", CASES)
def test_gemm_matches_gemv(qtype, rows, cols, m):
    torch = pytest.importorskip("torch")
    w = tm.Weight(qtype, rows, cols, synth.make_weights(qtype, rows, cols, seed=101))
    try:
        x = torch.from_numpy(synth.make_activations(cols, batch=m, seed=102)).cuda()
        x[5] *= 1000.0  # rows with their own scales
        x[7] = 0.0
        y = torch.full((m, rows), float("nan"), device="cuda")
        acc = torch.zeros((m, rows), dtype=torch.int64, device="cuda")
        w.gemm(x, y, m, row_acc=acc)
        if m <= 64:
            y_ref, acc_ref = per_row_gemv(w, x, m, rows)
        else:
            y_ref = torch.empty((m, rows), device="cuda")
            acc_ref = torch.zeros((m, rows), dtype=torch.int64, device="cuda")
            w.gemv(x, y_ref, batch=m, row_acc=acc_ref)
        torch.cuda.synchronize()
        assert tm.device_error(0) == 0
        assert torch.equal(acc, acc_ref)
        assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32))
    finally:
        w.free()


SKINNY = [(synth.Q4_K, 896, 4864, 16), (synth.Q6_K, 896, 4864, 16), (synth.Q5_0, 200, 96, 5),
          (synth.Q5_0, 1152, 896, 33), (synth.Q4_K, 896, 4864, 64), (synth.Q5_0, 4864, 896, 1)]


@pytest.mark.parametrize("qtype,rows,cols,m", SKINNY)
def test_skinny_split_k_matches_gemv(qtype, rows, cols, m):
    """m <= 64 rows: weights as the 128-row MMA operand, the batch as N, K split
    across CTAs with int64 partial sums in a workspace that the last CTA of each
    row tile drains and zeroes -- three calls in a row must all match."""
    torch = pytest.importorskip("torch")
    w = tm.Weight(qtype, rows, cols, synth.make_weights(qtype, rows, cols, seed=111))
    try:
        for call in range(3):
            x = torch.from_numpy(synth.make_activations(cols, batch=m, seed=112 + call)).cuda()
            if m > 3:
                x[3] *= 1000.0
                x[m - 1] = 0.0
            y = torch.full((m, rows), float("nan"), device="cuda")
            acc = torch.zeros((m, rows), dtype=torch.int64, device="cuda")
            w.gemm(x, y, m, row_acc=acc)
            y_ref, acc_ref = per_row_gemv(w, x, m, rows)
            # tmac_gemv at this batch (tensor cores from batch 8) agrees as well
            y_b = torch.empty((m, rows), device="cuda")
            w.gemv(x, y_b, batch=m)
            torch.cuda.synchronize()
            assert tm.device_error(0) == 0
            assert torch.equal(y_b.view(torch.int32), y_ref.view(torch.int32)), call
            assert torch.equal(acc, acc_ref), call
            assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32)), call
    finally:
        w.free()


@pytest.mark.parametrize("qtype,rows,cols,m", [(synth.Q8_0, 128, 896, 300), (synth.Q8_0, 200, 96, 129)])
def test_gemm_q8_0_matches_gemv(qtype, rows, cols, m):
    """NATIVE Q8_0 (the attn_v of the Q8_0 layers in prefill): one GEMM per
    64-column tile, folded into y in tile order exactly as the Q8_0 GEMV."""
    torch = pytest.importorskip("torch")
    w = tm.Weight(qtype, rows, cols, synth.make_weights(qtype, rows, cols, seed=111))
    try:
        x = torch.from_numpy(synth.make_activations(cols, batch=m, seed=112)).cuda()
        x[3] *= 300.0
        x[9] = 0.0
        y = torch.full((m, rows), float("nan"), device="cuda")
        w.gemm(x, y, m)
        y_ref = torch.empty((m, rows), device="cuda")
        w.gemv(x, y_ref, batch=m)
        torch.cuda.synchronize()
        assert tm.device_error(0) == 0
        assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32))
    finally:
        w.free()


@pytest.mark.parametrize("qtype,rows,cols", [(synth.Q5_0, 1152, 896), (synth.Q6_K, 896, 4864),
                                             (synth.Q4_K, 896, 4864), (synth.Q8_0, 128, 896)])
def test_gemm_rows_equal_the_oracle_at_prefill_size(qtype, rows, cols):
    """M = 1024 activation rows (a 2 x 512-token prefill slice); rows spread over
    the batch are checked directly against the oracle (the restated reference
    driver, oracle/tmac_oracle.c), y bit for bit and the int64 row sums."""
    import oracle
    torch = pytest.importorskip("torch")
    m = 1024
    raw = synth.make_weights(qtype, rows, cols, seed=121)
    w = tm.Weight(qtype, rows, cols, raw)
    try:
        xh = synth.make_activations(cols, batch=m, seed=122)
        xh[100] *= 1e4
        x = torch.from_numpy(xh).cuda()
        y = torch.empty((m, rows), device="cuda")
        acc = None if qtype == synth.Q8_0 else torch.zeros((m, rows), dtype=torch.int64, device="cuda")
        w.gemm(x, y, m, row_acc=acc)
        torch.cuda.synchronize()
        assert tm.device_error(0) == 0
        yc = y.cpu().numpy()
        ac = None if acc is None else acc.cpu().numpy()
        for r in (0, 100, 511, 777, 1023):
            o = oracle.gemv(qtype, raw, rows, cols, xh[r])
            np.testing.assert_array_equal(yc[r].view(np.int32), o.y.view(np.int32), err_msg=f"row {r}")
            if ac is not None:
                np.testing.assert_array_equal(ac[r], o.row_acc, err_msg=f"row {r}")
    finally:
        w.free()
