"""INT8 model parity: the CUDA INT8 forward (yb_cuda_set_int8 +
yb_cuda_forward) against the CPU INT8 oracle under the same scale table.  The
INT8 rules are integer once the scales are fixed, so every int8 stage tensor
and its per-channel scales must be bit-exact, and so must the dequantised
Detect logits (float(acc) * float(s_ref * s_w), one rounding on both sides);
the detections go through the same decode / sigmoid / top-k as the FP32 path
and are compared with its rules."""
import numpy as np
import pytest

from parity import compare_dets, dets_ok

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def calib(weights_n0):
    import yb_weights as yw
    from oracle import Oracle

    o = Oracle(weights_n0)
    return o, o.calibrate(yw.make_batch(range(1000, 1004), 96, 96))


@pytest.fixture(scope="module")
def model_i8(weights_n0, calib):
    import yolo_b200 as yb

    m = yb.Model(weights_n0)
    m.set_int8(calib[1])
    yield m
    m.close()


def _check_image(m, ref, image):
    for i, (name, (q, cs)) in enumerate(ref["stages"].items()):
        gq, gcs = m.int8_stage(i, image)
        assert gq.shape == q.shape, name
        assert np.array_equal(gcs, cs), name
        bad = np.argwhere(gq != q)
        assert bad.size == 0, (name, len(bad), bad[:4].tolist())


@pytest.mark.parametrize("hw", [(128, 128), (640, 640), (256, 320)])
def test_int8_bit_exact(model_i8, calib, hw):
    import yb_weights as yw

    o, scales = calib
    img = yw.make_input(2, *hw)
    got = model_i8.forward(img)
    logits, _ = model_i8.head(1)
    ref = o.forward_i8(img, scales, stages=True)
    assert len(ref["stages"]) == 23
    _check_image(model_i8, ref, 0)
    assert np.array_equal(logits[0], ref["logits"])
    c = compare_dets(got["dets"][0], ref["dets"])
    print(f"{hw}: dets {c}")
    assert dets_ok(c)


def test_int8_batch(model_i8, calib):
    """Images of a batch are independent: image i of a batch of 3 equals the oracle on image i."""
    import yb_weights as yw

    o, scales = calib
    imgs = yw.make_batch([21, 22, 23], 128, 160)
    got = model_i8.forward(imgs)["dets"]
    logits, _ = model_i8.head(3)
    for i in range(3):
        ref = o.forward_i8(imgs[i : i + 1], scales, stages=True)
        _check_image(model_i8, ref, i)
        assert np.array_equal(logits[i], ref["logits"]), i
        assert dets_ok(compare_dets(got[i], ref["dets"])), i


def test_int8_stage_dump_dequantised(model_i8, calib):
    """The stage callback of an INT8 forward reports q * scale per channel."""
    import yb_weights as yw

    img = yw.make_input(3, 96, 128)
    out = model_i8.forward(img, stages=True)
    for i in (0, 9, 11, 22):
        q, cs = model_i8.int8_stage(i)
        name = f"stage_{i + 1:02d}_buf{i}"
        want = q.astype(np.float32) * cs[:, None, None]
        assert np.array_equal(out["stages"][name][0], want), name


def test_precision_switch(weights_n0, calib):
    """FP32 -> INT8 -> FP32 on one context: each mode gives its own results."""
    import yb_weights as yw
    import yolo_b200 as yb

    o, scales = calib
    img = yw.make_input(4, 128, 128)
    m = yb.Model(weights_n0)
    try:
        f1 = m.forward(img)["dets"]
        m.set_int8(scales)
        q = m.forward(img)["dets"]
        lq, _ = m.head(1)
        assert np.array_equal(lq[0], o.forward_i8(img, scales)["logits"])
        m.set_int8(None)
        f2 = m.forward(img)["dets"]
        assert np.array_equal(f1, f2)
        assert not np.array_equal(f1, q)
        with pytest.raises(yb.YBError):
            m.int8_stage(0)
    finally:
        m.close()


def test_missing_scale_reported(weights_n0, calib):
    import yb_weights as yw
    import yolo_b200 as yb

    _, scales = calib
    partial = {k: v for k, v in scales.items() if k != "model.9.cv2"}
    m = yb.Model(weights_n0)
    try:
        m.set_int8(partial)
        with pytest.raises(yb.YBError, match="model.9.cv2"):
            m.forward(yw.make_input(5, 64, 64))
        with pytest.raises(yb.YBError):
            m.set_int8({"input": -1.0})
    finally:
        m.close()


def test_device_calibration(weights_n0, calib):
    """Device calibration (FP32 forwards with statistics) names the same
    tensors as the oracle's and lands within the FP32 path's tolerance of its
    scales; the INT8 forward under the device table is bit-exact with the
    oracle under the same table."""
    import yb_weights as yw
    import yolo_b200 as yb

    o, scales = calib
    m = yb.Model(weights_n0)
    try:
        dev = m.calibrate_int8(yw.make_batch(range(1000, 1004), 96, 96))
        assert set(dev) == set(scales)
        worst = max(abs(dev[k] - scales[k]) / scales[k] for k in scales)
        print(f"device vs oracle calibration: {len(dev)} scales, worst rel diff {worst:.2e}")
        assert worst < 1e-2
        img = yw.make_input(6, 160, 128)
        got = m.forward(img)
        lg, _ = m.head(1)
        ref = o.forward_i8(img, dev, stages=True)
        _check_image(m, ref, 0)
        assert np.array_equal(lg[0], ref["logits"])
        assert dets_ok(compare_dets(got["dets"][0], ref["dets"]))
    finally:
        m.close()


def test_int8_s_width(weights_s0):
    """The s width (channels x2: 4-head and 2-head attention, 32/64-channel
    patch-mode convolutions) under a device-calibrated table, bit-exact with
    the oracle under the same table."""
    import yb_weights as yw
    import yolo_b200 as yb
    from oracle import Oracle

    m = yb.Model(weights_s0)
    try:
        scales = m.calibrate_int8(yw.make_batch(range(1100, 1103), 128, 128))
        img = yw.make_input(8, 192, 256)
        got = m.forward(img)
        lg, _ = m.head(1)
        ref = Oracle(weights_s0).forward_i8(img, scales, stages=True)
        _check_image(m, ref, 0)
        assert np.array_equal(lg[0], ref["logits"])
        assert dets_ok(compare_dets(got["dets"][0], ref["dets"]))
    finally:
        m.close()


@pytest.mark.parametrize("hw", [(768, 768), (1216, 1280), (1280, 1536)])
def test_int8_long_attention(model_i8, calib, hw):
    """Key counts of the streamed-chunk attention kernel (512 < N <= 1920):
    576 (pass-1 chunks 256, 256, 64), 1520 (not a multiple of 64) and 1920
    (the largest); every stage bit-exact."""
    import yb_weights as yw

    o, scales = calib
    img = yw.make_input(11, *hw)
    model_i8.forward(img)
    lg, _ = model_i8.head(1)
    ref = o.forward_i8(img, scales, stages=True)
    _check_image(model_i8, ref, 0)
    assert np.array_equal(lg[0], ref["logits"])


def test_int8_1280(model_i8, calib):
    """1280 x 1280: attention over 1600 tokens (13 key blocks), bit-exact."""
    import yb_weights as yw

    o, scales = calib
    img = yw.make_input(9, 1280, 1280)
    got = model_i8.forward(img)
    lg, _ = model_i8.head(1)
    ref = o.forward_i8(img, scales, stages=True)
    _check_image(model_i8, ref, 0)
    assert np.array_equal(lg[0], ref["logits"])
    assert dets_ok(compare_dets(got["dets"][0], ref["dets"]))
