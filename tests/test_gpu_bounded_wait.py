"""The bounded barrier waits of the tcgen05 convolution, exercised without a
GPU fault: yb_conv_debug_withhold makes the next launch's producer warps arm
no barrier and issue no copy, with a 1 ms bound on every wait.  The UMMA
issuer's first wait runs out, the kernel records the wait error, drains,
frees its tensor memory and returns: yb_conv_check reports ERROR_DEVICE, and
the next launches of the same handle, and a model forward on the same
device, are clean and bit-equal to the ones before."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _split(x):
    import torch

    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    return torch.cat([hi.reshape(-1), lo.reshape(-1)])


@pytest.mark.parametrize("ci,co,k,hw", [(64, 64, 3, 40), (64, 128, 1, 32), (24, 40, 1, 17)])
def test_wait_runs_out_then_recovers(ci, co, k, hw, weights_n0):
    """Patch mode (3x3), TMA im2col (1x1, 64 channels) and the cp.async
    gather (24 channels): each mode's first wait is the one that runs out."""
    import torch

    import yb_weights as yw
    import yolo_b200 as yb

    L = yb.lib()
    m = yb.Model(weights_n0)
    img = yw.make_input(5, 128, 128)
    before = m.forward(img)["dets"]
    rng = np.random.default_rng(ci + co)
    w = (rng.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
    b = (rng.standard_normal(co) * 0.1).astype(np.float32)
    h = C.c_void_p()
    pad = (k - 1) // 2
    yb.check(L.yb_conv_create(0, w.ctypes.data, b.ctypes.data, co, ci, k, k, 1, pad, 1, C.byref(h)), "yb_conv_create")
    try:
        cip = L.yb_conv_ci_pad(h)
        B = 2
        x = torch.zeros((B, hw, hw, cip))
        x[..., :ci] = torch.from_numpy(rng.standard_normal((B, hw, hw, ci)).astype(np.float32))
        d_x = _split(x).cuda()
        cop = (co + 7) // 8 * 8
        n_out = 2 * B * hw * hw * cop

        def run():
            y = torch.zeros((n_out,), dtype=torch.bfloat16, device="cuda")
            torch.cuda.synchronize()
            yb.check(L.yb_conv_run(h, d_x.data_ptr(), B, hw, hw, y.data_ptr(), None), "yb_conv_run")
            return y

        y0 = run()
        yb.check(L.yb_conv_check(h), "yb_conv_check")
        yb.check(L.yb_conv_debug_withhold(h), "yb_conv_debug_withhold")
        run()
        st = L.yb_conv_check(h)
        msg = yb.last_error()
        print(f"{ci}->{co} {k}x{k}: withheld launch -> status {st} ({msg})")
        # The UMMA issuer's stage wait (code 1) or the epilogue's accumulator
        # wait (code 3) gives up first; both run under the same 1 ms bound.
        assert st == yb.ERROR_DEVICE
        assert "error code 1" in msg or "error code 3" in msg
        y1 = run()
        yb.check(L.yb_conv_check(h), "yb_conv_check")
        assert torch.equal(y0.cpu(), y1.cpu())
        after = m.forward(img)["dets"]
        assert np.array_equal(before, after)
    finally:
        yb.check(L.yb_conv_destroy(h), "yb_conv_destroy")
        m.close()


def test_first_layer_handle_has_no_waits():
    import yolo_b200 as yb

    L = yb.lib()
    w = np.zeros((16, 3, 3, 3), np.float32)
    h = C.c_void_p()
    yb.check(L.yb_conv_create(0, w.ctypes.data, None, 16, 3, 3, 3, 2, 1, 1, C.byref(h)), "yb_conv_create")
    try:
        assert L.yb_conv_debug_withhold(h) == yb.ERROR_NOT_IMPLEMENTED
    finally:
        L.yb_conv_destroy(h)
