"""The standalone layers.h / detect.h entry points that the model graph does
not call one by one (it fuses or folds them), each run on the GPU through the
C ABI against the reference's semantics:

  * silu_forward (layers.c:10-21): x / (1 + expf(-x)) in place;
  * pool2d_max_forward (layers.c:191-217): k x k window, padding k/2 excluded
    (-FLT_MAX start), any stride, output size from the output tensor;
  * upsample_nearest_forward (layers.c:23-39): nearest, integer scale;
  * dwconv3x3_same_forward (layers.c:269-290): depthwise 3x3, padding 1, bias
    first and taps in (ky, kx) order, batch 1;
  * detect_forward_one2one (detect.c:253-454): the Detect head on P3/P4/P5
    feature tensors, against the oracle's detections from the same features.

Pooling and upsampling are copies and must be exact; the arithmetic ones are
held to fp32 rounding (the device keeps activations as split bf16 pairs,
relative error <= 2^-17)."""
import ctypes as C

import numpy as np
import pytest

from parity import compare_dets, dets_ok

pytestmark = pytest.mark.gpu


def _tv(a):
    import yolo_b200 as yb

    return yb.tensor_view(np.ascontiguousarray(a, dtype=np.float32))


def _silu_ref(x):
    x = x.astype(np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


@pytest.mark.parametrize("shape", [(1, 16, 20, 20), (2, 24, 7, 9), (1, 8, 1, 1)])
def test_silu_forward(shape):
    import yolo_b200 as yb

    rng = np.random.default_rng(1)
    x = (rng.standard_normal(shape) * 4).astype(np.float32)
    x.flat[0] = 0.0
    t = _tv(x.copy())
    yb.check(yb.lib().silu_forward(C.byref(t)), "silu_forward")
    got = t._array
    want = _silu_ref(x)
    err = np.max(np.abs(got - want) / np.maximum(1.0, np.abs(want)))
    print(f"silu {shape}: max rel err {err:.2e}")
    assert err <= 2e-5
    assert got.flat[0] == 0.0


def _maxpool_ref(x, k, s, Ho, Wo):
    B, Cc, H, W = x.shape
    pad = k // 2
    out = np.full((B, Cc, Ho, Wo), -np.finfo(np.float32).max, np.float32)
    for oy in range(Ho):
        for ox in range(Wo):
            for ky in range(k):
                for kx in range(k):
                    iy, ix = oy * s - pad + ky, ox * s - pad + kx
                    if 0 <= iy < H and 0 <= ix < W:
                        out[:, :, oy, ox] = np.maximum(out[:, :, oy, ox], x[:, :, iy, ix])
    return out


@pytest.mark.parametrize("k,s,H,W", [(5, 1, 20, 20), (3, 2, 16, 16), (5, 1, 7, 11), (3, 1, 1, 1)])
def test_pool2d_max_forward(k, s, H, W):
    import yolo_b200 as yb

    rng = np.random.default_rng(2)
    x = rng.standard_normal((1, 16, H, W)).astype(np.float32)
    pad = k // 2
    Ho, Wo = (H + 2 * pad - k) // s + 1, (W + 2 * pad - k) // s + 1
    out = np.zeros((1, 16, Ho, Wo), np.float32)
    to = _tv(out)
    yb.check(yb.lib().pool2d_max_forward(C.byref(to), C.byref(_tv(x)), k, s), "pool2d_max_forward")
    assert np.array_equal(to._array, _maxpool_ref(x, k, s, Ho, Wo))


@pytest.mark.parametrize("scale,shape", [(2, (1, 16, 20, 20)), (2, (2, 8, 5, 3)), (3, (1, 8, 4, 4))])
def test_upsample_nearest_forward(scale, shape):
    import yolo_b200 as yb

    rng = np.random.default_rng(3)
    x = rng.standard_normal(shape).astype(np.float32)
    B, Cc, H, W = shape
    out = np.zeros((B, Cc, H * scale, W * scale), np.float32)
    to = _tv(out)
    yb.check(yb.lib().upsample_nearest_forward(C.byref(to), C.byref(_tv(x)), scale), "upsample_nearest_forward")
    want = x.repeat(scale, axis=2).repeat(scale, axis=3)
    assert np.array_equal(to._array, want)


def _dw_ref(x, w, b):
    """The reference's loop order in float32: s = bias, then s += x * w over
    (ky, kx), out-of-image taps skipped."""
    _, Cc, H, W = x.shape
    s = np.broadcast_to(b.reshape(1, Cc, 1, 1), x.shape).astype(np.float32).copy() if b is not None else \
        np.zeros_like(x)
    xp = np.zeros((1, Cc, H + 2, W + 2), np.float32)
    xp[:, :, 1:-1, 1:-1] = x
    valid = np.zeros((H + 2, W + 2), bool)
    valid[1:-1, 1:-1] = True
    for ky in range(3):
        for kx in range(3):
            tap = xp[:, :, ky : ky + H, kx : kx + W]
            ok = valid[ky : ky + H, kx : kx + W]
            prod = (tap * w[:, 0, ky, kx].reshape(1, Cc, 1, 1)).astype(np.float32)
            s = np.where(ok, (s + prod).astype(np.float32), s)
    return s


# Maps of 40 rows and more take 8-row strips per thread; ragged edges included.
@pytest.mark.parametrize("Cc,H,W,bias", [(16, 20, 20, True), (80, 13, 9, True), (8, 1, 5, False),
                                         (64, 80, 80, True), (80, 41, 43, True), (48, 40, 17, False)])
def test_dwconv3x3_same_forward(Cc, H, W, bias):
    import yolo_b200 as yb

    rng = np.random.default_rng(4)
    x = rng.standard_normal((1, Cc, H, W)).astype(np.float32)
    w = (rng.standard_normal((Cc, 1, 3, 3)) / 3).astype(np.float32)
    b = (rng.standard_normal(Cc) * 0.1).astype(np.float32) if bias else None
    out = np.zeros_like(x)
    to = _tv(out)
    st = yb.lib().dwconv3x3_same_forward(C.byref(to), C.byref(_tv(x)), C.byref(_tv(w)),
                                         C.byref(_tv(b)) if bias else None)
    yb.check(st, "dwconv3x3_same_forward")
    want = _dw_ref(x, w, b)
    err = float(np.max(np.abs(to._array - want) / np.maximum(1.0, np.abs(want))))
    print(f"dwconv {Cc}x{H}x{W}: max rel err {err:.2e}")
    # Inputs and outputs are split bf16 pairs (about 2^-17 relative each);
    # over the 409,600 outputs of the largest case the tail reaches 2.3e-5.
    assert err <= 3e-5


def test_detect_forward_one2one(weights_n0_soft):
    """model_create / model_load_weights (reference API), then the Detect head
    alone on the oracle's P3/P4/P5 stage tensors of a 640x640 image; the
    non-saturating weight set, so the ranking is decided by scores."""
    import yb_weights as yw
    import yolo_b200 as yb
    from oracle import Oracle

    L = yb.lib()
    img = yw.make_input(12, 640, 640)
    ref = Oracle(weights_n0_soft).forward(img, stages=True)
    feats = [ref["stages"][n] for n in ("stage_17_buf16", "stage_20_buf19", "stage_23_buf22")]
    m = yb.ModelT()
    yb.check(L.model_create(C.byref(m), 640, 640), "model_create")
    try:
        yb.check(L.model_load_weights(C.byref(m), weights_n0_soft.encode()), "model_load_weights")
        out = np.zeros((1, 300, 6, 1), np.float32)
        to = _tv(out)
        views = [_tv(f) for f in feats]
        yb.check(L.detect_forward_one2one(C.byref(m), 23, *[C.byref(v) for v in views], C.byref(to)),
                 "detect_forward_one2one")
        c = compare_dets(to._array.reshape(300, 6), ref["dets"])
        print(f"detect_forward_one2one: {c}")
        assert c["k"] == 300 and dets_ok(c) and c["matched"] >= 290
        # Any other module index is refused, as the device graph wires Detect at model.23.
        assert L.detect_forward_one2one(C.byref(m), 22, *[C.byref(v) for v in views], C.byref(to)) != 0
    finally:
        L.model_destroy(C.byref(m))
