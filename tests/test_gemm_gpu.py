"""Tensor-core batched matmul (tmac_gemm, prefill) against the GEMV.

tmac_gemm runs every activation row through the same arithmetic as one
tmac_gemv call (the reference's matmul_fpga_* per token), on tcgen05 int8 MMAs
over byte planes of the exact int16 weights.  Bar: y and the int64 row sums
identical to tmac_gemv with batch m, bit for bit, including partial tiles
(m and rows not multiples of 128) and K not a multiple of the 128-byte stage.
"""
import numpy as np
import pytest

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
        y_ref = torch.empty((m, rows), device="cuda")
        acc_ref = torch.zeros((m, rows), dtype=torch.int64, device="cuda")
        w.gemv(x, y_ref, batch=m, row_acc=acc_ref)
        torch.cuda.synchronize()
        assert tm.device_error(0) == 0
        assert torch.equal(acc, acc_ref)
        assert torch.equal(y.view(torch.int32), y_ref.view(torch.int32))
    finally:
        w.free()
