"""Multi-process image sharding on CPU (gloo, world size 2): shard bounds,
the host gather of per-rank detections, and a rank that fails before the
gather (the other rank must end with an error from the group timeout, not
hang).  No GPU work: the per-image "detections" are computed by the CPU
oracle's top-k on seeded predictions."""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _fake_dets(img):
    import sys

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from oracle import Oracle

    rng = np.random.default_rng(1000 + img)
    pred = rng.random((400, 84), dtype=np.float32)
    return Oracle.postprocess(pred, nc=80, max_det=300, cap=300)


def _worker(rank, world, port, B, mode, q):
    import datetime
    import sys

    sys.path[:0] = [os.path.join(ROOT, "yolo-baremetal_b200"), os.path.join(ROOT, "oracle")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    import yb_shard

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        b0, b1 = yb_shard.shard_bounds(B, world, rank)
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected host failure before the gather")
        local = np.stack([_fake_dets(i) for i in range(b0, b1)]) if b1 > b0 else np.zeros((0, 300, 6), np.float32)
        out = yb_shard.gather_detections(local, B)
        q.put((rank, "ok", out))
    except Exception as e:  # reported to the parent
        q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(B, mode):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, B, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(2):
        r, status, payload = q.get(timeout=120)
        res[r] = (status, payload)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_shard_bounds():
    import yb_shard

    for B in (0, 1, 7, 64):
        for G in (1, 2, 3, 8):
            spans = [yb_shard.shard_bounds(B, G, g) for g in range(G)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            assert all(spans[i][1] == spans[i + 1][0] for i in range(G - 1))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1
    with pytest.raises(ValueError):
        yb_shard.shard_bounds(4, 2, 2)


@pytest.mark.parametrize("B", [5, 8])
def test_gather_two_ranks(B):
    res = _run(B, "ok")
    want = np.stack([_fake_dets(i) for i in range(B)])
    for r in (0, 1):
        status, out = res[r]
        assert status == "ok", out
        assert np.array_equal(out, want)


def test_failed_rank_surfaces_as_error():
    res = _run(6, "fail")
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error"  # the survivor's gather ends with an error instead of hanging
