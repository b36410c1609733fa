"""yb_cuda_forward_sharded: the image-sharded multi-GPU forward (no collective;
one context and host thread per shard).  With one visible GPU the shards are
two independent contexts on that GPU, which exercises the same host logic.
The deadline path is driven from the host (a shard thread that sleeps before
it starts), so no kernel is made to fail."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def shard_models(weights_n0):
    import torch

    import yolo_b200 as yb

    devs = [0, 1] if torch.cuda.device_count() >= 2 else [0, 0]
    ms = [yb.Model(weights_n0, device=d) for d in devs]
    yield ms
    for m in ms:
        m.close()


def test_sharded_equals_single_context(shard_models):
    import yb_weights as yw
    import yolo_b200 as yb

    imgs = yw.make_batch([31, 32, 33, 34, 35], 160, 192)
    st, dets = yb.forward_sharded(shard_models, imgs, timeout_ms=60000)
    yb.check(st, "yb_cuda_forward_sharded")
    single = shard_models[0].forward(imgs)["dets"]
    assert np.array_equal(dets, single)


def test_sharded_deadline_reports_timeout_then_recovers(shard_models):
    import yb_weights as yw
    import yolo_b200 as yb

    imgs = yw.make_batch([41, 42], 128, 128)
    L = yb.lib()
    yb.check(L.yb_cuda_debug_inject_stall(shard_models[1].ctx, 1500), "inject stall")
    try:
        st, _ = yb.forward_sharded(shard_models, imgs, timeout_ms=300)
        assert st == yb.ERROR_TIMEOUT, st
        assert "deadline" in yb.last_error()
    finally:
        yb.check(L.yb_cuda_debug_inject_stall(shard_models[1].ctx, 0), "clear stall")
    st, dets = yb.forward_sharded(shard_models, imgs, timeout_ms=60000)
    yb.check(st, "yb_cuda_forward_sharded after timeout")
    assert np.array_equal(dets, shard_models[0].forward(imgs)["dets"])


def test_sharded_across_all_gpus_timed(weights_n0):
    """The benchmark's global batch of 64 640x640 images split over every
    visible GPU by yb_cuda_forward_sharded (detections land in one host
    array), bit-equal to one GPU's forward of the same batch; prints the
    wall-clock images/s of both (skipped with one GPU)."""
    import time

    import torch

    import yb_weights as yw
    import yolo_b200 as yb

    G = torch.cuda.device_count()
    if G < 2:
        pytest.skip("one GPU visible")
    ms = [yb.Model(weights_n0, device=d) for d in range(G)]
    try:
        imgs = yw.make_batch(range(1, 65), 640, 640)
        st, dets = yb.forward_sharded(ms, imgs, timeout_ms=60000)
        yb.check(st, "yb_cuda_forward_sharded")
        one = ms[0].forward(imgs)["dets"]
        assert np.array_equal(dets, one)
        reps = 5
        t0 = time.perf_counter()
        for _ in range(reps):
            yb.check(yb.forward_sharded(ms, imgs, timeout_ms=60000)[0], "sharded")
        ts = (time.perf_counter() - t0) / reps
        t0 = time.perf_counter()
        for _ in range(reps):
            ms[0].forward(imgs)
        t1 = (time.perf_counter() - t0) / reps
        print(f"64 images: {G} GPUs sharded {64 / ts:.0f} images/s ({1e3 * ts:.1f} ms), "
              f"1 GPU {64 / t1:.0f} images/s ({1e3 * t1:.1f} ms), host buffers")
    finally:
        for m in ms:
            m.close()


def test_batch_size_does_not_change_fp32_results(shard_models):
    """The benchmark batch of 64 640x640 images through one host forward
    (16-image plans, pipelined) and as two 32-image shards (32-image plans,
    whose small 20x20 layers get narrower N tiles): bit-equal detections.
    Every FP32 convolution sums the same products in the same order whatever
    its N tiling, so the batch size never changes a result."""
    import yb_weights as yw
    import yolo_b200 as yb

    imgs = yw.make_batch(range(101, 165), 640, 640)
    st, dets = yb.forward_sharded(shard_models, imgs, timeout_ms=60000)
    yb.check(st, "yb_cuda_forward_sharded")
    single = shard_models[0].forward(imgs)["dets"]
    assert np.array_equal(dets, single)
