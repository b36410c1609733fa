"""Streaming forwards (yb_cuda_forward_submit / _rgb8_submit / _wait) through
the C ABI: batches queued two at a time give exactly the detections of the
synchronous calls on the same inputs (same kernels, same plan shapes), in
FP32 and INT8; finished and unknown tickets; a precision switch with
batches in flight finishes them first."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _pinned(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()


def _stream(m, batches, H, W, rgb8=False, sh=0, sw=0):
    """Submits every batch with at most two in flight; returns their outputs."""
    import torch

    outs = [torch.full((b.shape[0], 300, 6), float("nan")).pin_memory() for b in batches]
    tickets = []
    for x, o in zip(batches, outs):
        if rgb8:
            t = m.submit_rgb8(x.data_ptr(), x.shape[0], sh, sw, o.data_ptr(), H, W)
        else:
            t = m.submit(x.data_ptr(), x.shape[0], H, W, o.data_ptr())
        tickets.append(t)
        if len(tickets) > 2:
            m.wait(tickets[-3])
    for t in tickets:
        m.wait(t)
    return [o.numpy() for o in outs]


def test_stream_matches_sync(weights_n0):
    import yb_weights as yw
    import yolo_b200 as yb

    H = W = 256
    m = yb.Model(weights_n0)
    try:
        batches = [yw.make_batch(range(10 * i, 10 * i + 4), H, W) for i in range(5)]
        want = [m.forward(b)["dets"] for b in batches]
        got = _stream(m, [_pinned(b) for b in batches], H, W)
        for g, w in zip(got, want):
            assert np.array_equal(g, w)
        # Finished tickets return at once; unknown ones are an error.
        x0, o0 = _pinned(batches[0]), _pinned(np.zeros((4, 300, 6), np.float32))
        t = m.submit(x0.data_ptr(), 4, H, W, o0.data_ptr())
        m.wait(t)
        assert np.array_equal(o0.numpy(), want[0])
        m.wait(t)
        with pytest.raises(yb.YBError):
            m.wait(t + 100)
    finally:
        m.close()


def test_stream_rgb8_matches_sync(weights_n0):
    import yolo_b200 as yb

    rng = np.random.default_rng(5)
    sh, sw, H, W = 300, 400, 256, 320
    m = yb.Model(weights_n0)
    try:
        frames = [rng.integers(0, 256, size=(3, sh, sw, 3), dtype=np.uint8) for _ in range(4)]
        want = [m.forward_rgb8(f, H, W) for f in frames]
        got = _stream(m, [_pinned(f) for f in frames], H, W, rgb8=True, sh=sh, sw=sw)
        for g, w in zip(got, want):
            assert np.array_equal(g, w)
    finally:
        m.close()


def test_stream_int8_and_precision_switch(weights_n0):
    import torch

    import yb_weights as yw
    import yolo_b200 as yb

    H = W = 128
    m = yb.Model(weights_n0)
    try:
        scales = m.calibrate_int8(yw.make_batch(range(1, 5), H, W), apply=False)
        batches = [yw.make_batch(range(40 + 3 * i, 43 + 3 * i), H, W) for i in range(3)]
        want32 = [m.forward(b)["dets"] for b in batches]
        m.set_int8(scales)
        want8 = [m.forward(b)["dets"] for b in batches]
        got8 = _stream(m, [_pinned(b) for b in batches], H, W)
        for g, w in zip(got8, want8):
            assert np.array_equal(g, w)
        # Two INT8 batches in flight, then back to FP32: both finish first
        # with their INT8 results, and the next streamed batch is FP32.
        xs = [_pinned(b) for b in batches[:2]]
        outs = [torch.zeros((3, 300, 6)).pin_memory() for _ in range(2)]
        ts = [m.submit(x.data_ptr(), 3, H, W, o.data_ptr()) for x, o in zip(xs, outs)]
        m.set_int8(None)
        for t in ts:
            m.wait(t)
        for o, w in zip(outs, want8[:2]):
            assert np.array_equal(o.numpy(), w)
        got32 = _stream(m, [_pinned(batches[2])], H, W)
        assert np.array_equal(got32[0], want32[2])
    finally:
        m.close()
