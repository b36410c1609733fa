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
