"""tmac_gemv_static: the block-quant GEMV whose x_q / x_scale scratch is a fixed
module-scope array (no device allocation).  Two calls in a row on one stream
must each equal tmac_gemv on the same inputs bit for bit; sizes above the fixed
scratch are rejected with TMAC_ERR_SHAPE.  Named to be collected last, and
self-contained so that it also passes alone."""
import ctypes

import numpy as np
import pytest

import tmac_zynq_fpga_b200 as tm
from tmac_zynq_fpga_b200 import synth

pytestmark = pytest.mark.gpu

MAX_VALUES = 131072  # TMAC_STATIC_MAX_VALUES
MAX_BATCH = 64       # TMAC_STATIC_MAX_BATCH


def _static(w, x, y, batch, stream=None):
    return tm.lib().tmac_gemv_static(w.handle, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                     batch, stream)


# The last case fills the scratch exactly (batch 64 x 2048 columns = the value
# limit, and the batch limit), through four 16-vector launches.
@pytest.mark.parametrize("qtype,rows,cols,batch", [(synth.Q5_0, 4864, 896, 1), (synth.Q5_0, 896, 896, 16),
                                                   (synth.Q4_K, 896, 4864, 1), (synth.Q6_K, 896, 4864, 4),
                                                   (synth.Q5_0, 896, 2048, 64)])
def test_static_matches_gemv_two_calls(qtype, rows, cols, batch):
    torch = pytest.importorskip("torch")
    w = tm.Weight(qtype, rows, cols, synth.make_weights(qtype, rows, cols, seed=91))
    try:
        xs = [torch.from_numpy(synth.make_activations(cols, batch, seed=92 + i) * (1 + 3 * i)).cuda()
              for i in range(2)]
        outs = []
        for x in xs:  # two calls in a row, then compare each
            y = torch.full((batch, rows), float("nan"), device="cuda")
            assert _static(w, x, y, batch) == 0, tm.lib().tmac_last_error()
            outs.append(y)
        for x, y in zip(xs, outs):
            ref = torch.empty((batch, rows), device="cuda")
            w.gemv(x, ref, batch)
            torch.cuda.synchronize()
            assert torch.equal(y.view(torch.int32), ref.view(torch.int32))
    finally:
        w.free()


def test_static_rejects_oversize_and_unsupported():
    torch = pytest.importorskip("torch")
    cols = 4864
    w = tm.Weight(synth.Q4_K, 256, cols, synth.make_weights(synth.Q4_K, 256, cols, seed=93))
    q5 = tm.Weight(synth.Q5_0, 64, 896, synth.make_weights(synth.Q5_0, 64, 896, seed=95))
    q8 = tm.Weight(synth.Q8_0, 64, 896, synth.make_weights(synth.Q8_0, 64, 896, seed=94))
    try:
        big = MAX_VALUES // cols + 1
        x = torch.zeros((big, cols), device="cuda")
        y = torch.zeros((big, 256), device="cuda")
        assert _static(w, x, y, big) == -3 and b"exceeds" in tm.lib().tmac_last_error()
        x2 = torch.zeros((MAX_BATCH + 1, 896), device="cuda")
        y2 = torch.zeros((MAX_BATCH + 1, 64), device="cuda")
        assert _static(q5, x2, y2, MAX_BATCH + 1) == -3  # batch above the scale slots
        assert _static(q8, x2, y2, 1) == -2              # Q8_0 uses no scratch
    finally:
        w.free()
        q5.free()
        q8.free()
