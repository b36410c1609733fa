"""The device-resident FP32 convolution handle (yb_conv_create / yb_conv_run),
which times the isolated convolution sweep, against a float64 PyTorch
convolution of the same values (conv2d_forward + bias + SiLU semantics,
layers.c:41-90) on the five sweep shapes and on shapes that take the other
operand modes.  The device keeps activations as split bf16 pairs (hi + lo,
relative representation error <= 2^-17) and multiplies them as three bf16
products with fp32 accumulation, so each output is held to 1e-4 of the
output's largest magnitude."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [  # (ci, co, k, stride, hw): the sweep, then other modes
    (3, 16, 3, 2, 640), (16, 32, 3, 2, 320), (64, 64, 1, 1, 160), (128, 128, 3, 1, 40), (256, 256, 3, 1, 20),
    (32, 64, 3, 1, 24), (24, 40, 1, 1, 17), (48, 96, 3, 2, 33),
]


def to_split(x_nhwc):
    """fp32 torch NHWC -> flat bf16 [hi plane, lo plane] and the exact value hi + lo."""
    import torch

    hi = x_nhwc.to(torch.bfloat16)
    lo = (x_nhwc - hi.float()).to(torch.bfloat16)
    return torch.cat([hi.reshape(-1), lo.reshape(-1)]), hi.float() + lo.float()


def from_split(buf, shape):
    n = int(np.prod(shape))
    return (buf[:n].float() + buf[n:].float()).reshape(shape)


@pytest.mark.parametrize("ci,co,k,stride,hw", SHAPES)
def test_conv_handle_matches_float64(ci, co, k, stride, hw):
    import torch

    import yolo_b200 as yb

    L = yb.lib()
    B = 2
    pad = (k - 1) // 2
    rng = np.random.default_rng(ci * 7 + co)
    w = (rng.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
    b = (rng.standard_normal(co) * 0.1).astype(np.float32)
    h = C.c_void_p()
    yb.check(L.yb_conv_create(0, w.ctypes.data, b.ctypes.data, co, ci, k, k, stride, pad, 1, C.byref(h)),
             "yb_conv_create")
    try:
        cip = L.yb_conv_ci_pad(h)
        x = torch.from_numpy(rng.standard_normal((B, ci, hw, hw)).astype(np.float32))
        if cip == 0:  # NCHW fp32 input (first-layer kernel)
            d_x = x.cuda()
            xv = x.double()
        else:
            xp = torch.zeros((B, hw, hw, cip))
            xp[..., :ci] = x.permute(0, 2, 3, 1)
            d_x, val = to_split(xp)
            d_x = d_x.cuda()
            xv = val[..., :ci].permute(0, 3, 1, 2).double()
        ho = (hw + 2 * pad - k) // stride + 1
        cop = (co + 7) // 8 * 8
        d_y = torch.full((2 * B * ho * ho * cop,), float("nan"), dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
        yb.check(L.yb_conv_run(h, d_x.data_ptr(), B, hw, hw, d_y.data_ptr(), None), "yb_conv_run")
        yb.check(L.yb_conv_check(h), "yb_conv_check")
        got = from_split(d_y.cpu(), (B, ho, ho, cop))[..., :co].permute(0, 3, 1, 2).double()
        ref = torch.nn.functional.conv2d(xv, torch.from_numpy(w).double(), torch.from_numpy(b).double(),
                                         stride=stride, padding=pad)
        ref = ref * torch.sigmoid(ref)
        err = float((got - ref).abs().max() / ref.abs().max())
        print(f"{ci}->{co} {k}x{k} s{stride} @{hw}: rel err {err:.2e} (ci_pad {cip})")
        assert err <= 1e-4
    finally:
        yb.check(L.yb_conv_destroy(h), "yb_conv_destroy")


def test_conv_handle_rejects_bad_shapes():
    import yolo_b200 as yb

    L = yb.lib()
    w = np.zeros((16, 8, 5, 5), np.float32)
    h = C.c_void_p()
    assert L.yb_conv_create(0, w.ctypes.data, None, 16, 8, 5, 5, 1, 2, 1, C.byref(h)) == yb.ERROR_INVALID_DIMS
    assert not h.value
