"""Greedy top-1 over logits on the GPU (tmac_gemv_top1 / tmac_top1): the
packed key must name the oracle's first maximum of the bit-exact logits."""
import numpy as np
import pytest

import oracle
import tmac_zynq_fpga_b200 as tm
from tmac_zynq_fpga_b200 import shard, synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qtype,rows,cols,base", [(tm.Q8_0, 151936, 896, 0), (tm.Q8_0, 18992, 896, 56976),
                                                  (tm.Q8_0, 100, 96, 5), (tm.Q5_0, 4864, 896, 0),
                                                  (tm.Q6_K, 896, 4864, 3)])
def test_gemv_top1_matches_oracle(qtype, rows, cols, base):
    raw = synth.make_weights(qtype, rows, cols, seed=rows % 97)
    x = synth.make_activations(cols, batch=2, seed=rows % 89)
    w = tm.Weight(qtype, rows, cols, raw)
    xt = torch.from_numpy(x).cuda()
    y = torch.empty((2, rows), dtype=torch.float32, device="cuda")
    key = torch.full((2,), -1, dtype=torch.int64, device="cuda")
    w.gemv_top1(xt, y, key, index_base=base, batch=2)
    torch.cuda.synchronize()
    assert tm.device_error(0) == 0
    for b in range(2):
        o = oracle.gemv(qtype, raw, rows, cols, x[b])
        np.testing.assert_array_equal(y[b].cpu().numpy().view(np.int32), o.y.view(np.int32))
        val, idx = tm.top1_decode(key[b].item())
        assert idx == base + shard.top1_index(o.y)
        assert np.float32(val) == o.y.max()
        assert int(key[b].item()) == int(shard.pack_keys(o.y, base).max())
    w.free()


def test_top1_ties_pick_lowest_index_and_merge():
    y = torch.full((5000,), -3.0, device="cuda")
    y[4000] = 7.0
    y[1234] = 7.0
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    tm.check(tm.lib().tmac_top1(y.data_ptr(), 2500, 0, key.data_ptr(), None))
    tm.check(tm.lib().tmac_top1(y[2500:].data_ptr(), 2500, 2500, key.data_ptr(), None))
    torch.cuda.synchronize()
    assert tm.top1_decode(key.item()) == (7.0, 1234)
