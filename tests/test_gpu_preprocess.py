"""Device preprocess (yb_cuda_preprocess_rgb8 / yb_cuda_forward_rgb8) against
the CPU restatement of the reference's preprocessing, which is pinned to the
reference bit for bit (test_preprocess_host.py): the network input must be
bit-identical, so the forward from 8-bit images must equal the forward of the
oracle-preprocessed fp32 input exactly."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [(480, 640, 640, 640), (720, 1280, 640, 640), (37, 100, 96, 64), (640, 640, 640, 640), (1, 1, 32, 32),
          (7, 5, 1, 1), (333, 211, 160, 224)]


def _rgb(B, sh, sw, seed):
    return np.random.default_rng(seed).integers(0, 256, size=(B, sh, sw, 3), dtype=np.uint8)


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("sh,sw,oh,ow", SHAPES)
def test_device_preprocess_bit_exact(mode, sh, sw, oh, ow):
    import torch

    import yolo_b200 as yb
    from oracle import Oracle

    rgb = _rgb(2, sh, sw, sh + sw + mode)
    d_rgb = torch.from_numpy(rgb).cuda()
    d_out = torch.full((2, 3, oh, ow), -1.0, dtype=torch.float32, device="cuda")
    yb.check(yb.lib().yb_cuda_preprocess_rgb8(d_rgb.data_ptr(), 2, sh, sw, mode, d_out.data_ptr(), oh, ow, None),
             "yb_cuda_preprocess_rgb8")
    torch.cuda.synchronize()
    want = Oracle.preprocess(rgb, oh, ow, mode)
    got = d_out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("mode", [0, 1])
def test_forward_rgb8_equals_forward(weights_n0, mode):
    import yolo_b200 as yb
    from oracle import Oracle

    m = yb.Model(weights_n0)
    try:
        rgb = _rgb(3, 360, 480, 40 + mode)
        dets8 = m.forward_rgb8(rgb, 320, 320, resize=mode)
        lg8, bx8 = m.head(3)
        x = Oracle.preprocess(rgb, 320, 320, mode)
        dets = m.forward(x)["dets"]
        lg, bx = m.head(3)
        assert np.array_equal(dets8, dets)
        assert np.array_equal(lg8, lg) and np.array_equal(bx8, bx)
        # INT8 mode through the same entry point
        m.calibrate_int8(x)
        q8 = m.forward_rgb8(rgb, 320, 320, resize=mode)
        qf = m.forward(x)["dets"]
        assert np.array_equal(q8, qf)
    finally:
        m.close()
