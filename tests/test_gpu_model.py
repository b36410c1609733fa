"""Full-model parity: the CUDA forward (yb_cuda_forward / model_forward_ex)
against the CPU oracle on seeded random-init YOLO26 weights and seeded U[0,1)
inputs, stage by stage, on the pre-sigmoid class logits, and on the top-k
detections."""
import numpy as np
import pytest

from parity import LOGIT_ATOL, STAGE_RTOL, compare_dets, dets_ok, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model_n0(weights_n0):
    import yolo_b200 as yb

    m = yb.Model(weights_n0)
    yield m
    m.close()


def _oracle(path):
    from oracle import Oracle

    return Oracle(path)


@pytest.mark.parametrize("hw", [640, 128])
def test_stages_logits_dets(model_n0, weights_n0, hw):
    import yb_weights as yw

    img = yw.make_input(1, hw, hw)
    got = model_n0.forward(img, stages=True)
    logits, boxes = model_n0.head(1)
    ref = _oracle(weights_n0).forward(img, stages=True)
    worst = 0.0
    for name, want in ref["stages"].items():
        if name.startswith("stage_24") or name.startswith("stage_25"):
            continue
        have = got["stages"][name]
        assert have.shape == want.shape, name
        e = rel_err(have, want)
        worst = max(worst, e)
        print(f"{name}: rel err {e:.2e}")
        assert e <= STAGE_RTOL, name
    lerr = float(np.max(np.abs(logits[0] - ref["logits"])))
    print(f"logits max abs err {lerr:.3e} (max |logit| {np.abs(ref['logits']).max():.1f}); worst stage {worst:.2e}")
    assert lerr <= LOGIT_ATOL
    c = compare_dets(got["dets"][0], ref["dets"])
    print(f"dets: {c}")
    assert dets_ok(c)


def test_dets_non_saturating(weights_n0_soft):
    """With scores below saturation the ranking is decided by scores: the
    detections must match row for row."""
    import yb_weights as yw
    import yolo_b200 as yb

    m = yb.Model(weights_n0_soft)
    img = yw.make_input(7, 640, 640)
    got = m.forward(img)["dets"][0]
    ref = _oracle(weights_n0_soft).forward(img)["dets"]
    c = compare_dets(got, ref)
    print(f"soft weights dets: {c}")
    assert c["k"] == 300 and dets_ok(c) and c["matched"] >= 290
    m.close()


def test_batch_equals_single(model_n0):
    """Images are independent: a batch of 3 gives each image's B=1 result bit for bit."""
    import yb_weights as yw

    imgs = yw.make_batch([11, 12, 13], 256, 320)
    batch = model_n0.forward(imgs)["dets"]
    for i in range(3):
        single = model_n0.forward(imgs[i : i + 1])["dets"][0]
        assert np.array_equal(batch[i], single), i


def test_pipelined_batch_equals_device_batch(model_n0):
    """A host batch of 48 runs as three pipelined 16-image sub-batches; it gives
    the same detections as the one-plan device forward of the same 48 images,
    bit for bit, and keeps no head tensors."""
    import torch

    import yb_weights as yw

    B, H, W = 48, 128, 160
    imgs = yw.make_batch(range(100, 100 + B), H, W)
    piped = model_n0.forward(imgs)["dets"]
    with pytest.raises(RuntimeError):
        model_n0.head(B)
    d_in = torch.from_numpy(imgs).cuda()
    d_out = torch.empty((B, 300, 6), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    model_n0.forward_device(d_in.data_ptr(), d_out.data_ptr(), B, H, W)
    torch.cuda.synchronize()
    dev = d_out.cpu().numpy()
    for i in range(B):
        assert np.array_equal(piped[i], dev[i]), i


def test_repeatable(model_n0):
    import yb_weights as yw

    img = yw.make_input(3, 320, 320)
    a = model_n0.forward(img)["dets"]
    b = model_n0.forward(img)["dets"]
    assert np.array_equal(a, b)


def test_profile_steps(model_n0):
    import yb_weights as yw

    out = model_n0.forward(yw.make_input(1, 640, 640), profile=True)
    ms = out["step_ms"]
    assert len(ms) == 25 and all(v >= 0 for v in ms)
    assert ms[0] > 0 and ms[23] > 0


def test_s_width_model(weights_s0):
    """The width-0.5 (s) model: widths come from the weights, same kernels."""
    import yb_weights as yw
    import yolo_b200 as yb

    m = yb.Model(weights_s0)
    img = yw.make_input(5, 256, 256)
    got = m.forward(img, stages=True)
    logits, _ = m.head(1)
    ref = _oracle(weights_s0).forward(img, stages=True)
    for name, want in ref["stages"].items():
        if name.startswith("stage_2") and name >= "stage_24":
            continue
        assert rel_err(got["stages"][name], want) <= STAGE_RTOL, name
    assert float(np.max(np.abs(logits[0] - ref["logits"]))) <= LOGIT_ATOL
    m.close()


def test_detect_cv2_cv3_fallback(weights_n0_o2m):
    """Without one2one_cv2/cv3 in the checkpoint the Detect head runs the
    one-to-many cv2/cv3 branches (detect.c:297-299): FP32 stages, logits and
    detections against the oracle, and the INT8 forward bit-exact with the
    INT8 oracle under the same table."""
    import yb_weights as yw
    import yolo_b200 as yb

    o = _oracle(weights_n0_o2m)
    img = yw.make_input(14, 320, 320)
    m = yb.Model(weights_n0_o2m)
    try:
        got = m.forward(img)
        logits, _ = m.head(1)
        ref = o.forward(img)
        assert float(np.max(np.abs(logits[0] - ref["logits"]))) <= LOGIT_ATOL
        c = compare_dets(got["dets"][0], ref["dets"])
        print(f"cv2/cv3 FP32 dets: {c}")
        assert dets_ok(c) and c["matched"] >= 290
        scales = m.calibrate_int8(yw.make_batch(range(1300, 1303), 128, 128))
        q = m.forward(img)["dets"][0]
        lq, _ = m.head(1)
        rq = o.forward_i8(img, scales)
        assert np.array_equal(lq[0], rq["logits"])
        assert dets_ok(compare_dets(q, rq["dets"]))
    finally:
        m.close()
