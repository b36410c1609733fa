"""yb_cuda_detect_topk_noalloc, the top-k entry point that allocates nothing,
called through the C ABI on head tensors from a full forward and compared
with that forward's own detections (yb_cuda_forward), on two calls in a row,
then once more on a side stream with the device's free memory unchanged.
The file name sorts last so the test also runs after every other GPU test in
the same process; it passes alone as well."""
import numpy as np
import pytest

from parity import compare_dets, dets_ok

pytestmark = pytest.mark.gpu


def test_detect_topk_noalloc_matches_forward(weights_n0):
    import torch

    import yb_weights as yw
    import yolo_b200 as yb

    L = yb.lib()
    B, H, W, K = 2, 320, 256, 300
    m = yb.Model(weights_n0)
    try:
        imgs = yw.make_batch([21, 22], H, W)
        want = m.forward(imgs, max_det=K)["dets"]
        logits, boxes = m.head(B)
        N, nc = logits.shape[1], logits.shape[2]
        d_logits = torch.from_numpy(logits).cuda()
        d_boxes = torch.from_numpy(boxes).cuda()
        outs = []
        for _ in range(2):
            d_dets = torch.full((B, K, 6), float("nan"), dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            yb.check(L.yb_cuda_detect_topk_noalloc(d_logits.data_ptr(), d_boxes.data_ptr(), B, N, nc, K,
                                                   d_dets.data_ptr(), None), "yb_cuda_detect_topk_noalloc")
            torch.cuda.synchronize()
            outs.append(d_dets.cpu().numpy())
        # Once the first call on the device has run, a call on another stream
        # leaves the device's free memory unchanged: nothing is allocated.
        side = torch.cuda.Stream()
        d_dets = torch.full((B, K, 6), float("nan"), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        yb.check(L.yb_cuda_detect_topk_noalloc(d_logits.data_ptr(), d_boxes.data_ptr(), B, N, nc, K,
                                               d_dets.data_ptr(), side.cuda_stream), "yb_cuda_detect_topk_noalloc")
        side.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        assert free1 == free0, (free0, free1)
        outs.append(d_dets.cpu().numpy())
        for got in outs:
            for i in range(B):
                c = compare_dets(got[i], want[i])
                print(f"image {i}: {c}; bit-exact {np.array_equal(got[i], want[i])}")
                assert dets_ok(c) and c["k"] == min(K, N)
        assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
        # Sizes beyond the scratch array are refused before any launch.
        st = L.yb_cuda_detect_topk_noalloc(d_logits.data_ptr(), d_boxes.data_ptr(), 1 << 20, 2, nc, K,
                                           d_dets.data_ptr(), None)
        assert st == yb.ERROR_INVALID_DIMS
        assert "scratch capacity" in yb.last_error()
        assert L.yb_cuda_detect_topk_noalloc(None, d_boxes.data_ptr(), B, N, nc, K, d_dets.data_ptr(),
                                             None) == yb.ERROR_NULL_POINTER
    finally:
        m.close()
