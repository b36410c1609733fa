"""Fused block kernels against the unfused graph.

Every Bottleneck of the C3k2 / C3k blocks whose 3x3 convolutions map
C -> CM -> C channels with (C, CM) = (16, 16), (32, 32), (32, 16) or
(16, 8) (layers.c:92-108 with the shortcut) runs as one launch whose
intermediate stays in shared memory (bottleneck_tc.cu), and the two 1x1
convolutions of each C3k that read the same input (layers.c:156-189) run as
one launch with the output channels of both.  K order, split products and
epilogue arithmetic are those of the separate convolution launches, so the
forward must be bit-identical with fusion on and off: every stage tensor,
the pre-sigmoid logits, the decoded boxes and the detections.  The oracle
parity of the fused graph is covered by the model tests, which run with
fusion on (the default)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _n_ops(m, B, H, W):
    import yolo_b200 as yb

    n = C.c_int()
    yb.check(yb.lib().yb_cuda_profile_ops(m.ctx, B, H, W, 300, 0, None, 0, C.byref(n)), "yb_cuda_profile_ops")
    return n.value


def _run(m, img):
    B = img.shape[0]
    out = m.forward(img, stages=B == 1)
    logits, boxes = m.head(B)
    return out, logits, boxes


@pytest.mark.parametrize("B,H,W", [(1, 640, 640), (3, 256, 320), (2, 96, 160), (1, 64, 96)])
def test_fused_bitwise_equal(weights_n0, B, H, W):
    import yb_weights as yw
    import yolo_b200 as yb

    m = yb.Model(weights_n0)
    try:
        img = yw.make_input(B, H, W)
        m.set_fusion(False)
        a, la, ba = _run(m, img)
        n_off = _n_ops(m, B, H, W)
        m.set_fusion(True)
        b, lb, bb = _run(m, img)
        n_on = _n_ops(m, B, H, W)
        print(f"B{B} {H}x{W}: {n_off} launches unfused, {n_on} fused")
        # YOLO26n: the two C3k bottlenecks of model.6, .13 (32 channels),
        # .16 (16) and .19 (32) and the e = 0.5 Bottlenecks of model.2
        # (16 -> 8 -> 16) and model.4 (32 -> 16 -> 32) are fused (10
        # launches fewer), and the cv1 / cv2 pair of each of the five C3k
        # blocks (model.6, .8, .13, .16, .19) is one launch (5 fewer).
        assert n_off - n_on == 15
        if B == 1:
            assert a["stages"].keys() == b["stages"].keys()
            for k in sorted(a["stages"]):
                x, y = a["stages"][k], b["stages"][k]
                if not np.array_equal(x, y):
                    d = np.abs(x - y)
                    idx = np.unravel_index(np.argmax(d), d.shape)
                    print(f"{k}: {np.count_nonzero(d)} of {d.size} differ, max {d.max():.3e} at {idx} "
                          f"(scale {np.abs(x).max():.3e})")
            for k in a["stages"]:
                assert np.array_equal(a["stages"][k], b["stages"][k]), k
        assert np.array_equal(la, lb)
        assert np.array_equal(ba, bb)
        assert np.array_equal(a["dets"], b["dets"])
    finally:
        m.close()


def test_fused_s_width(weights_s0):
    """s width: the 32-channel bottlenecks (model.2, model.16's C3k) fuse,
    the 64-channel ones stay separate launches; bit-identical either way."""
    import yb_weights as yw
    import yolo_b200 as yb

    m = yb.Model(weights_s0)
    try:
        img = yw.make_input(2, 192, 256)
        m.set_fusion(False)
        a, la, _ = _run(m, img)
        m.set_fusion(True)
        b, lb, _ = _run(m, img)
        assert np.array_equal(a["dets"], b["dets"])
        assert np.array_equal(la, lb)
    finally:
        m.close()


def test_fused_int8_bitwise_equal(weights_n0):
    """INT8 graph: the Bottlenecks run as bottleneck_i8_kernel (kind::i8,
    the int8 intermediate in shared memory); every int8 stage tensor, the
    dequantised logits and the detections are identical with fusion on and
    off, and switching fusion rebuilds the plans of the streaming path."""
    import yb_weights as yw
    import yolo_b200 as yb

    m = yb.Model(weights_n0)
    try:
        img = yw.make_input(2, 256, 320)
        scales = m.calibrate_int8(yw.make_batch(range(1000, 1002), 96, 96), apply=False)
        m.set_int8(scales)
        m.set_fusion(False)
        a = m.forward(img)["dets"]
        la, _ = m.head(2)
        sa = [m.int8_stage(i)[0] for i in range(23)]
        n_off = _n_ops(m, 2, 256, 320)
        m.set_fusion(True)
        b = m.forward(img)["dets"]
        lb, _ = m.head(2)
        sb = [m.int8_stage(i)[0] for i in range(23)]
        n_on = _n_ops(m, 2, 256, 320)
        print(f"INT8: {n_off} launches unfused, {n_on} fused")
        # The ten Bottlenecks of model.2, .4, .6, .13, .16 and .19.
        assert n_off - n_on == 10
        for i in range(23):
            assert np.array_equal(sa[i], sb[i]), i
        assert np.array_equal(la, lb)
        assert np.array_equal(a, b)
        m.set_int8(None)
        ref = m.forward(img)["dets"]
        m.set_fusion(False)
        assert np.array_equal(m.forward(img)["dets"], ref)
    finally:
        m.close()
