"""GPU parity: every GEMV path of libtmac_cuda.so against the oracle, which is
itself pinned to the reference's compiled CPU code (test_oracle_pin.py).
Bar: y bit-identical, int64 row and per-unit sums identical."""
import numpy as np
import pytest

import oracle
import tmac_zynq_fpga_b200 as tm
from tmac_zynq_fpga_b200 import synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

PATH = {tm.MODE_NATIVE: oracle.PATH_NATIVE, tm.MODE_INT16: oracle.PATH_INT16, tm.MODE_F32: oracle.PATH_F32}


def run_gpu(w, x, batch):
    xt = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    y = torch.empty((batch, w.rows), dtype=torch.float32, device="cuda")
    ra = ua = None
    if w.mode != tm.MODE_F32:
        ra = torch.zeros((batch, w.rows), dtype=torch.int64, device="cuda")
        ua = torch.zeros((batch, w.rows, max(w.units, 1)), dtype=torch.int64, device="cuda")
    w.gemv(xt, y, batch=batch, row_acc=ra, unit_acc=ua)
    torch.cuda.synchronize()
    assert tm.device_error(w.device) == 0
    return (y.cpu().numpy(), None if ra is None else ra.cpu().numpy(),
            None if ua is None else ua.cpu().numpy())


def check_case(qtype, rows, cols, mode=tm.MODE_NATIVE, batch=1, seed=0, row_max_abs=None, weights=None, x=None):
    raw = synth.make_weights(qtype, rows, cols, seed=seed) if weights is None else weights
    if x is None:
        x = synth.make_activations(cols, batch=batch, seed=seed)
    w = tm.Weight(qtype, rows, cols, raw, mode=mode, row_max_abs=row_max_abs)
    y, ra, ua = run_gpu(w, x, batch)
    for b in range(batch):
        o = oracle.gemv(qtype, raw, rows, cols, x[b], path=PATH[mode], row_max_abs=row_max_abs)
        np.testing.assert_array_equal(y[b].view(np.int32), o.y.view(np.int32),
                                      err_msg=f"y bits differ (batch {b})")
        if ra is not None:
            np.testing.assert_array_equal(ra[b], o.row_acc, err_msg="int64 row sums differ")
            np.testing.assert_array_equal(ua[b][:, :w.units], o.unit_acc, err_msg="int64 unit sums differ")
    w.free()


@pytest.mark.parametrize("rows", [8, 64, 128, 896, 4864])
def test_q5_0_native(rows):
    check_case(tm.Q5_0, rows, 896)


def test_q5_0_batch():
    check_case(tm.Q5_0, 136, 896, batch=5, seed=3)


@pytest.mark.parametrize("rows,cols", [(32, 64), (33, 96), (130, 896), (128, 896), (1000, 896), (64, 2048)])
def test_q8_0_native(rows, cols):
    check_case(tm.Q8_0, rows, cols, seed=rows)


def test_q8_0_row_max_abs():
    rows, cols = 200, 896
    raw = synth.make_weights(tm.Q8_0, rows, cols, seed=7)
    rma = np.abs(np.random.default_rng(1).normal(0, 0.02, rows)).astype(np.float32) * 3
    rma[5] = 0.0  # below the 1e-10 floor -> row_scale 1
    check_case(tm.Q8_0, rows, cols, weights=raw, row_max_abs=rma)


def test_q8_0_logits_full():
    """Config 2 shape: 151936 x 896 (all 4748 row groups)."""
    check_case(tm.Q8_0, 151936, 896, seed=0)


@pytest.mark.parametrize("qtype", [tm.Q4_K, tm.Q6_K])
@pytest.mark.parametrize("rows,cols,batch", [(56, 256, 1), (32, 512, 2), (896, 4864, 1), (896, 4864, 16)])
def test_kquant_native(qtype, rows, cols, batch):
    check_case(qtype, rows, cols, batch=batch, seed=rows + batch)


@pytest.mark.parametrize("qtype,cols", [(tm.Q5_0, 896), (tm.Q8_0, 896), (tm.Q4_K, 512), (tm.Q6_K, 512),
                                        (tm.F32, 100), (tm.F16, 96)])
def test_int16_fallback(qtype, cols):
    check_case(qtype, 70, cols, mode=tm.MODE_INT16, batch=2, seed=11)


@pytest.mark.parametrize("qtype,cols", [(tm.Q5_0, 896), (tm.Q8_0, 896), (tm.Q4_K, 512), (tm.Q6_K, 512),
                                        (tm.F32, 100)])
def test_f32_path(qtype, cols):
    check_case(qtype, 50, cols, mode=tm.MODE_F32, seed=5)


@pytest.mark.parametrize("qtype,cols", [(tm.Q5_0, 896), (tm.Q8_0, 896), (tm.Q4_K, 512), (tm.Q6_K, 512)])
def test_zero_weights_and_activations(qtype, cols):
    """max < 1e-10 floors: row_inv / row_scale = 1 and x_scale = 1."""
    rows = 40
    raw = synth.make_weights(qtype, rows, cols, seed=2)
    raw2 = raw.copy()
    nbytes = len(raw) // rows
    raw2[:3 * nbytes] = 0  # first three rows: d = 0 / quants 0
    x = synth.make_activations(cols, batch=2, seed=2)
    x[1] = 0.0
    check_case(qtype, rows, cols, weights=raw2, x=x, batch=2)
    check_case(qtype, rows, cols, weights=raw2, x=x, batch=2, mode=tm.MODE_INT16)


def test_typed_entry_points_reject_mismatch():
    raw = synth.make_weights(tm.Q5_0, 8, 896)
    w = tm.Weight(tm.Q5_0, 8, 896, raw)
    x = torch.zeros(896, device="cuda")
    y = torch.zeros(8, device="cuda")
    rc = tm.lib().tmac_gemv_q8_0(w.handle, x.data_ptr(), y.data_ptr(), 1, None)
    assert rc == -2
    assert tm.lib().tmac_gemv_q5_0(w.handle, x.data_ptr(), y.data_ptr(), 1, None) == 0
    torch.cuda.synchronize()


def test_drop_in_matmul_switch():
    """The reference's matmul() dispatch: switched type -> core path, others -> INT16, none -> FP32."""
    A = tm.Tensor("blk.0.attn_q.weight", 64, 896, tm.Q5_0, synth.make_weights(tm.Q5_0, 64, 896, seed=9))
    x = synth.make_activations(896, seed=9)[0]
    for argv, path in ((["--fpga-q5-0"], oracle.PATH_NATIVE), (["--fpga-q8"], oracle.PATH_INT16),
                       ([], oracle.PATH_F32)):
        sw = tm.Switches().parse(argv)
        y = np.zeros(64, np.float32)
        tm.matmul(A, x, y, 64, 896, sw)
        o = oracle.gemv(tm.Q5_0, A.data, 64, 896, x, path=path)
        np.testing.assert_array_equal(y.view(np.int32), o.y.view(np.int32))


@pytest.mark.parametrize("qtype,rows,cols,batch", [(tm.Q5_0, 4864, 896, 1), (tm.Q5_0, 128, 896, 3),
                                                   (tm.Q8_0, 151936, 896, 1), (tm.Q8_0, 128, 896, 2),
                                                   (tm.Q4_K, 896, 4864, 1), (tm.Q6_K, 896, 4864, 16)])
def test_quantize_once_matches_gemv(qtype, rows, cols, batch):
    """tmac_quantize_x + tmac_gemv_xq == tmac_gemv bit for bit (the reference
    quantises x the same way in every driver, so sharing x_q changes nothing)."""
    raw = synth.make_weights(qtype, rows, cols, seed=17)
    x = synth.make_activations(cols, batch=batch, seed=17)
    w = tm.Weight(qtype, rows, cols, raw)
    xt = torch.from_numpy(x).cuda()
    xq = torch.empty((batch, cols), dtype=torch.int16, device="cuda")
    xs = torch.empty(batch, dtype=torch.float32, device="cuda")
    y1 = torch.empty((batch, rows), dtype=torch.float32, device="cuda")
    y2 = torch.empty_like(y1)
    tm.check(tm.lib().tmac_quantize_x(xt.data_ptr(), cols, batch, xq.data_ptr(), xs.data_ptr(), None))
    tm.check(tm.lib().tmac_gemv_xq(w.handle, xq.data_ptr(), xs.data_ptr(), y2.data_ptr(), batch, None))
    w.gemv(xt, y1, batch=batch)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y1.cpu().numpy().view(np.int32), y2.cpu().numpy().view(np.int32))
    for b in range(batch):
        xs_o, xq_o = oracle.quantize_x(x[b])
        assert np.float32(xs[b].item()) == xs_o
        np.testing.assert_array_equal(xq[b].cpu().numpy(), xq_o)
    w.free()


@pytest.mark.parametrize("qtype,rows,cols,batch", [(tm.Q4_K, 896, 4864, 16), (tm.Q6_K, 896, 4864, 8),
                                                   (tm.Q5_0, 4864, 896, 64), (tm.Q5_0, 200, 96, 9)])
def test_tensor_core_batches_equal_the_oracle(qtype, rows, cols, batch):
    """Batches of 8..64 without per-unit sums run on the tensor cores (split-K
    tcgen05 kernel); y and the int64 row sums must still equal the oracle."""
    raw = synth.make_weights(qtype, rows, cols, seed=rows + batch)
    x = synth.make_activations(cols, batch=batch, seed=batch)
    w = tm.Weight(qtype, rows, cols, raw)
    try:
        xt = torch.from_numpy(x).cuda()
        y = torch.empty((batch, rows), dtype=torch.float32, device="cuda")
        ra = torch.zeros((batch, rows), dtype=torch.int64, device="cuda")
        w.gemv(xt, y, batch=batch, row_acc=ra)
        torch.cuda.synchronize()
        assert tm.device_error(w.device) == 0
        y, ra = y.cpu().numpy(), ra.cpu().numpy()
        for b in range(0, batch, max(1, batch // 4)):
            o = oracle.gemv(qtype, raw, rows, cols, x[b], path=oracle.PATH_NATIVE)
            np.testing.assert_array_equal(y[b].view(np.int32), o.y.view(np.int32), err_msg=f"y bits differ (batch {b})")
            np.testing.assert_array_equal(ra[b], o.row_acc, err_msg="int64 row sums differ")
    finally:
        w.free()
