"""The Detect top-k (detect_postprocess_from_pred, detect.c:63-166) on crafted
class logits, through yb_cuda_detect_topk_noalloc, against the oracle's
postprocess of the same scores.

Logits drawn from {-200, 0, 100} have the sigmoid values 0, 0.5 and 1 exactly
(on the host and on the device), so the scores are massive ties and the
expected detections are bit-exact: equal scores keep ascending anchor order in
stage 1 and ascending (slot, class) order in stage 2.  The two densities of
100s drive both stage-2 paths: few exact-1 pairs (ranked among the pairs that
can still make the cut) and many (the full radix select).  A continuous case
checks the same path on distinct scores within the score tolerance."""
import numpy as np
import pytest

from parity import compare_dets, dets_ok

pytestmark = pytest.mark.gpu


def _sig(x):
    return (1.0 / (1.0 + np.exp(-x.astype(np.float64)))).astype(np.float32)


def _run(logits, boxes, K):
    import torch

    import yolo_b200 as yb

    L = yb.lib()
    B, N, nc = logits.shape
    d_logits = torch.from_numpy(np.ascontiguousarray(logits)).cuda()
    d_boxes = torch.from_numpy(np.ascontiguousarray(boxes)).cuda()
    d_dets = torch.full((B, K, 6), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    yb.check(L.yb_cuda_detect_topk_noalloc(d_logits.data_ptr(), d_boxes.data_ptr(), B, N, nc, K,
                                           d_dets.data_ptr(), None), "yb_cuda_detect_topk_noalloc")
    torch.cuda.synchronize()
    return d_dets.cpu().numpy()


def _want(logits, boxes, probs, K):
    from oracle import Oracle

    B, N, nc = logits.shape
    out = []
    for b in range(B):
        pred = np.concatenate([boxes[b], probs[b]], axis=1)
        out.append(Oracle.postprocess(pred, nc, K, K))
    return np.stack(out)


@pytest.mark.parametrize("p100", [0.004, 0.1])
def test_topk_exact_ties(p100):
    rng = np.random.default_rng(7)
    B, N, nc, K = 3, 2100, 80, 300
    choice = rng.choice(3, size=(B, N, nc), p=[0.5, 0.5 - p100, p100])
    logits = np.array([-200.0, 0.0, 100.0], dtype=np.float32)[choice]
    probs = np.array([0.0, 0.5, 1.0], dtype=np.float32)[choice]
    assert np.array_equal(_sig(logits), probs)
    boxes = rng.uniform(0, 640, size=(B, N, 4)).astype(np.float32)
    got = _run(logits, boxes, K)
    want = _want(logits, boxes, probs, K)
    assert np.array_equal(got, want)


def test_topk_continuous_scores():
    rng = np.random.default_rng(8)
    B, N, nc, K = 2, 8400, 80, 300
    logits = rng.normal(-4.0, 2.0, size=(B, N, nc)).astype(np.float32)
    boxes = rng.uniform(0, 640, size=(B, N, 4)).astype(np.float32)
    got = _run(logits, boxes, K)
    want = _want(logits, boxes, _sig(logits), K)
    for b in range(B):
        c = compare_dets(got[b], want[b])
        assert dets_ok(c), c
