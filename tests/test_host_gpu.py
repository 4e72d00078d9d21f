"""tmac_gemv_host: the drop-in for the reference's matmul_fpga_* calls on host
arrays (sim/tmac_gguf.cpp:948-1085 and siblings).  y must equal the device
GEMV bit for bit whether y is pageable (staged through device memory) or
page-locked (for Q8_0 the kernel stores it straight into host memory)."""
import ctypes

import numpy as np
import pytest

import tmac_zynq_fpga_b200 as tm
from tmac_zynq_fpga_b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qtype,rows,cols,batch", [(synth.Q8_0, 151936, 896, 1), (synth.Q8_0, 4864, 896, 3),
                                                   (synth.Q5_0, 4864, 896, 2)])
@pytest.mark.parametrize("pinned", [False, True])
def test_gemv_host_matches_device(qtype, rows, cols, batch, pinned):
    w = tm.Weight(qtype, rows, cols, synth.make_weights(qtype, rows, cols, seed=13))
    x = synth.make_activations(cols, batch=batch, seed=14)
    ref = torch.empty((batch, rows), device="cuda")
    w.gemv(torch.from_numpy(x).cuda(), ref, batch=batch)
    torch.cuda.synchronize()
    xh = torch.from_numpy(x.copy())
    yh = torch.full((batch, rows), float("nan"))
    if pinned:
        xh, yh = xh.pin_memory(), yh.pin_memory()
    for _ in range(2):  # twice: the second call reuses the staging / the mapping
        tm.check(tm.lib().tmac_gemv_host(w.handle, ctypes.c_void_p(xh.data_ptr()), ctypes.c_void_p(yh.data_ptr()),
                                         batch))
        assert tm.device_error(0) == 0
        np.testing.assert_array_equal(yh.numpy().view(np.int32), ref.cpu().numpy().view(np.int32))
