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


@pytest.mark.parametrize("rows,cap", [(300, 100), (300, 7), (45, 100), (33, 0)])
def test_device_detection_lists(rows, cap):
    """yb_cuda_detections (batched decode_detections) against the oracle's
    restatement, which is pinned to the reference: scores equal to the
    threshold, NaN scores, capacity overflow."""
    import torch

    import yolo_b200 as yb
    from oracle import Oracle

    thr = np.float32(0.25)
    rng = np.random.default_rng(rows + cap)
    d = rng.standard_normal((3, rows, 6)).astype(np.float32) * 100
    d[..., 4] = rng.choice([thr, np.nextafter(thr, np.float32(1)), 0.0, 0.9, -1.0, np.nan], size=(3, rows))
    d[..., 5] = rng.integers(0, 80, (3, rows)).astype(np.float32)
    dd = torch.from_numpy(d).cuda()
    out = torch.zeros((3, max(cap, 1) * 6), dtype=torch.int32, device="cuda")
    cnt = torch.full((3,), -1, dtype=torch.int32, device="cuda")
    yb.check(yb.lib().yb_cuda_detections(dd.data_ptr(), 3, rows, thr, cap, out.data_ptr(), cnt.data_ptr(), None),
             "yb_cuda_detections")
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(Oracle.DET_DTYPE).reshape(3, -1)
    counts = cnt.cpu().numpy()
    for b in range(3):
        want, n = Oracle.decode_detections(d[b], thr, cap)
        assert counts[b] == n
        assert got[b, :n].tobytes() == want[:n].tobytes()


def test_get_detections_after_forward(weights_n0_soft):
    import yb_weights as yw
    import yolo_b200 as yb
    from oracle import Oracle

    m = yb.Model(weights_n0_soft)
    try:
        x = yw.make_batch([51, 52], 256, 256)
        dets = m.forward(x)["dets"]
        lists, counts = m.detections(2, threshold=0.5, capacity=50)
        for b in range(2):
            want, n = Oracle.decode_detections(dets[b], np.float32(0.5), 50)
            assert counts[b] == n
            assert lists[b, :n].tobytes() == want[:n].tobytes()
    finally:
        m.close()
