"""Device-side weight preparation (yb_cuda_load_bin_device) against the host
path (yb_cuda_load_bin) on the same converter .bin: the BatchNorm fold
(utils.c:81-106, model.c:121-180), the packed FP32 tcgen05 operand images in
every N tiling the graph uses, and the INT8 quantisation and packing under
one scale table must be bit-identical, and so must the forwards.  The
prepared-weight blob (yb_cuda_save_prepared / yb_cuda_load_prepared) must
restore the same images and results."""
import os
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _prefixes(path):
    import yb_weights as yw

    _, sd = yw.read_bin(path)
    convs, plain = [], []
    for k, v in sd.items():
        if v.ndim != 4 or v.shape[1] == 1:
            continue
        if k.endswith(".conv.weight"):
            convs.append(k[: -len(".conv.weight")])
        elif k.endswith(".weight") and not k.endswith(".bn.weight"):
            plain.append(k[: -len(".weight")])
    return convs, plain


@pytest.fixture(scope="module")
def pair(weights_n0):
    import yolo_b200 as yb

    t0 = time.perf_counter()
    host = yb.Model(weights_n0, prep="host")
    t1 = time.perf_counter()
    dev = yb.Model(weights_n0, prep="device")
    t2 = time.perf_counter()
    print(f"load: host preparation {1e3 * (t1 - t0):.1f} ms, device preparation {1e3 * (t2 - t1):.1f} ms")
    yield host, dev
    host.close()
    dev.close()


def test_fold_bit_identical(pair, weights_n0):
    host, dev = pair
    convs, plain = _prefixes(weights_n0)
    n = 0
    for p in convs:
        for t in (".conv.weight", ".conv.bias"):
            assert host.weight_image(p + t, 0) == dev.weight_image(p + t, 0), p + t
            n += 1
    for p in plain:
        assert host.weight_image(p + ".weight", 0) == dev.weight_image(p + ".weight", 0), p
    print(f"{n} folded tensors bit-identical")


def test_fp32_packing_bit_identical(pair, weights_n0):
    import yb_weights as yw

    host, dev = pair
    convs, plain = _prefixes(weights_n0)
    _, sd = yw.read_bin(weights_n0)
    n = 0
    for p in convs + plain:
        w = sd.get(p + ".conv.weight", sd.get(p + ".weight"))
        if w.shape[1] % 8:  # the first layer runs in the stem kernel, unpacked
            continue
        tiles = [0] + ([64, 128] if w.shape[0] >= 128 else [])
        for nt in tiles:
            a, b = host.weight_image(p, 1, nt), dev.weight_image(p, 1, nt)
            assert len(a) > 0 and a == b, (p, nt)
            n += 1
    print(f"{n} packed FP32 operand images bit-identical")


def test_forwards_and_int8_packing_identical(pair, weights_n0):
    import yb_weights as yw

    host, dev = pair
    img = yw.make_input(3, 320, 320)
    a, b = host.forward(img), dev.forward(img)
    assert np.array_equal(a["dets"], b["dets"])
    scales = host.calibrate_int8(yw.make_batch(range(1000, 1004), 128, 128))
    dev.set_int8(scales)
    qa, qb = host.forward(img), dev.forward(img)
    la, _ = host.head(1)
    lb, _ = dev.head(1)
    assert np.array_equal(la, lb)
    assert np.array_equal(qa["dets"], qb["dets"])
    for i in range(23):
        assert np.array_equal(host.int8_stage(i)[0], dev.int8_stage(i)[0]), i
    convs, plain = _prefixes(weights_n0)
    n = 0
    for p in convs + plain:
        # model.0 is quantised into the INT8 stem kernel's own layout; the
        # one-to-many Detect branches are not wired when one2one exists.
        if p == "model.0" or p.startswith("model.23.cv2.") or p.startswith("model.23.cv3."):
            continue
        x, y = host.weight_image(p, 2), dev.weight_image(p, 2)
        assert len(x) > 0 and x == y, p
        n += 1
    print(f"INT8: logits, detections and 23 stage tensors identical; {n} packed INT8 images bit-identical")
    host.set_int8(None)
    dev.set_int8(None)


def test_prepared_blob_roundtrip(pair, weights_n0, tmp_path):
    import yb_weights as yw
    import yolo_b200 as yb

    _, dev = pair
    blob = str(tmp_path / "yolo26n.prep")
    dev.save_prepared(blob)
    t0 = time.perf_counter()
    m = yb.Model(blob, prep="blob")
    print(f"blob {os.path.getsize(blob) / 1e6:.1f} MB, load {1e3 * (time.perf_counter() - t0):.1f} ms")
    try:
        convs, _ = _prefixes(weights_n0)
        for p in convs[1:]:
            assert m.weight_image(p, 1) == dev.weight_image(p, 1), p
        img = yw.make_input(4, 256, 256)
        assert np.array_equal(m.forward(img)["dets"], dev.forward(img)["dets"])
    finally:
        m.close()
    with open(str(tmp_path / "bad.prep"), "wb") as f:
        f.write(b"not a blob")
    with pytest.raises(yb.YBError):
        yb.Model(str(tmp_path / "bad.prep"), prep="blob")
