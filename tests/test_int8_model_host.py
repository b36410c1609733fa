"""CPU checks of the INT8 model oracle (our restatement; the reference has no
INT8 code): calibration covers every scale the INT8 graph needs, and the INT8
forward, dequantised, tracks the FP32 oracle within int8 quantisation error
stage by stage (a structural error -- wrong channels, scales or wiring --
shows up as errors of order 1)."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def int8_run(weights_n0):
    import yb_weights as yw
    from oracle import Oracle

    o = Oracle(weights_n0)
    scales = o.calibrate(yw.make_batch(range(1000, 1004), 96, 96))
    img = yw.make_input(1, 96, 96)
    return o, scales, o.forward_i8(img, scales, stages=True), o.forward(img, stages=True)


def test_calibration_names(int8_run):
    _, scales, _, _ = int8_run
    assert "input" in scales and "model.10.m.0.attn.ope" in scales and "model.22.m.0.1.ffn.1" in scales
    assert "model.2.m.0.cv2" in scales and "model.2.m.0.cv2:pre" in scales and "model.9.cv2" in scales
    assert all(v > 0 for v in scales.values())


def test_int8_tracks_fp32(int8_run):
    _, _, r8, rf = int8_run
    assert len(r8["stages"]) == 23
    for name, (q, cs) in r8["stages"].items():
        f = rf["stages"][name][0]
        err = np.abs(q.astype(np.float32) * cs[:, None, None] - f).max() / np.abs(f).max()
        assert err < 0.25, (name, err)
    lerr = np.abs(r8["logits"] - rf["logits"]).max() / np.abs(rf["logits"]).max()
    assert lerr < 0.15, lerr
