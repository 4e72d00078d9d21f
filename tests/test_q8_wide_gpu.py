"""GPU parity of the tensor-core Q8_0 GEMV (tall matrices: rows >= 16384,
128 <= cols <= 896), chosen at registration when TMAC_Q8_WIDE=1.  Same bar
as every GEMV path: y bit-identical to the oracle, int64 row sums and 64-column tile sums identical (sim/tmac_gguf.cpp:948-1085).  The
shapes cover ragged last row groups, a partial last 128-column k-block, an odd
block count (a last tile of one 32-column block), the 896-column maximum,
batches, a supplied row_max_abs and the top-1 key."""
import numpy as np
import pytest

import oracle
import tmac_zynq_fpga_b200 as tm
from tmac_zynq_fpga_b200 import synth

from test_gemv_gpu import check_case

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def wide_layout(monkeypatch):
    monkeypatch.setenv("TMAC_Q8_WIDE", "1")


@pytest.mark.parametrize("rows,cols,batch", [(16384, 896, 1), (20000, 896, 1), (16500, 800, 1), (17000, 736, 1),
                                             (16384, 864, 1), (16511, 128, 1), (20000, 896, 3),
                                             (151936, 896, 1)])
def test_q8_wide_matches_oracle(rows, cols, batch):
    check_case(tm.Q8_0, rows, cols, batch=batch, seed=rows + cols)


def test_q8_wide_row_max_abs_and_extreme_activations():
    rows, cols = 16640, 896
    raw = synth.make_weights(tm.Q8_0, rows, cols, seed=5)
    rma = np.abs(np.random.default_rng(1).normal(0, 1, rows)).astype(np.float32) + 0.5
    x = synth.make_activations(cols, batch=2, seed=6)
    x[0] *= 1e4
    x[1, :] = 0.0
    x[1, 17] = -3.0  # one non-zero activation
    check_case(tm.Q8_0, rows, cols, batch=2, weights=raw, row_max_abs=rma, x=x)


def test_q8_wide_top1_and_repeat():
    rows, cols = 40000, 896
    raw = synth.make_weights(tm.Q8_0, rows, cols, seed=9)
    w = tm.Weight(tm.Q8_0, rows, cols, raw)
    for step in range(3):
        x = synth.make_activations(cols, seed=20 + step) * (1 + 10 * step)
        xt = torch.from_numpy(x).cuda()
        y = torch.empty(rows, device="cuda")
        key = torch.zeros(1, dtype=torch.int64, device="cuda")
        w.gemv_top1(xt, y, key, index_base=123)
        torch.cuda.synchronize()
        assert tm.device_error(0) == 0
        o = oracle.gemv(tm.Q8_0, raw, rows, cols, x)
        np.testing.assert_array_equal(y.cpu().numpy().view(np.int32), o.y.view(np.int32))
        assert tm.top1_decode(key.item())[1] == 123 + int(np.argmax(o.y))
