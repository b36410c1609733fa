"""INT8 convolution on the tensor cores (yb_int8_conv_*, tcgen05 kind::i8)
against the CPU INT8 oracle, bit for bit: the five backbone shapes of the conv
sweep and edge shapes (channel padding, N tiles, two N tiles, odd maps,
batches, no activation, no bias)."""
import ctypes as C

import numpy as np
import pytest

from int8_util import conv_oracle, make_layer, ptr, quantize_lib

pytestmark = pytest.mark.gpu

# (ci, co, k, stride, H, W, B, act, bias)
SWEEP = [(3, 16, 3, 2, 640, 640, 1, True, True), (16, 32, 3, 2, 320, 320, 1, True, True),
         (64, 64, 1, 1, 160, 160, 1, True, True), (128, 128, 3, 1, 40, 40, 1, True, True),
         (256, 256, 3, 1, 20, 20, 1, True, True)]
EDGE = [(40, 48, 3, 1, 23, 17, 2, True, True), (32, 16, 3, 1, 80, 80, 1, False, True),
        (96, 272, 1, 1, 20, 24, 3, True, False), (64, 80, 3, 2, 33, 31, 2, True, True),
        (8, 16, 1, 1, 9, 7, 1, False, False), (200, 128, 3, 1, 12, 12, 1, True, True)]


def _run_gpu(lyr, q, k, stride):
    import torch

    import yolo_b200 as yb

    L = yb.lib()
    co, ci = q["wq"].shape[0], q["wq"].shape[1]
    h = C.c_void_p()
    yb.check(L.yb_int8_conv_create(0, ptr(q["wq"]), ptr(q["bq"]), ptr(q["mult"]), ptr(q["shift"]), ptr(q["lut"]),
                                   co, ci, k, k, stride, lyr["pad"], C.byref(h)), "yb_int8_conv_create")
    try:
        cp = L.yb_int8_conv_ci_pad(h)
        B, H, W, _ = lyr["xq"].shape
        x = torch.zeros((B, H, W, cp), dtype=torch.int8, device="cuda")
        x[..., :ci] = torch.from_numpy(lyr["xq"]).cuda()
        Ho, Wo = (H + 2 * lyr["pad"] - k) // stride + 1, (W + 2 * lyr["pad"] - k) // stride + 1
        y = torch.full((B, Ho, Wo, co), 99, dtype=torch.int8, device="cuda")
        torch.cuda.synchronize()
        yb.check(L.yb_int8_conv_run(h, x.data_ptr(), B, H, W, y.data_ptr(), None), "yb_int8_conv_run")
        yb.check(L.yb_int8_conv_check(h), "yb_int8_conv_check")
        return y.cpu().numpy()
    finally:
        L.yb_int8_conv_destroy(h)


@pytest.mark.parametrize("ci,co,k,stride,H,W,B,act,bias", SWEEP + EDGE)
def test_int8_conv_bit_exact(ci, co, k, stride, H, W, B, act, bias):
    lyr = make_layer(ci, co, k, H, W, B=B, seed=ci * 7 + co + H, act=act, bias=bias)
    q = quantize_lib(lyr)
    got = _run_gpu(lyr, q, k, stride)
    want = conv_oracle(lyr["xq"], q, k, stride, lyr["pad"])
    diff = np.count_nonzero(got != want)
    sat = np.mean(np.abs(want.astype(np.int32)) == 127)
    print(f"int8 conv {ci}->{co} k{k} s{stride} @{H}x{W} B{B}: {diff} of {want.size} differ; "
          f"{sat:.2%} saturated, {np.mean(want == 0):.2%} zero")
    assert diff == 0


@pytest.mark.parametrize("shrink", [2e-3, 1e-4])
def test_int8_conv_wide_requant(shrink):
    """Output scales far below the accumulator scale push requantisation
    shifts under 32, which the kernel serves with its 64-bit arithmetic
    instead of the 32-bit word path; results stay bit-exact."""
    lyr = make_layer(32, 48, 3, 20, 18, B=2, seed=5, act=False, bias=True)
    lyr["s_pre"] = lyr["s_out"] = np.float32(lyr["s_out"] * shrink)
    q = quantize_lib(lyr)
    assert int(q["shift"].min()) < 32
    got = _run_gpu(lyr, q, 3, 1)
    want = conv_oracle(lyr["xq"], q, 3, 1, lyr["pad"])
    assert np.count_nonzero(got != want) == 0
