"""The CPU restatement of the reference's image preprocessing (oracle,
preprocess_oracle.c) against the reference's own static functions, compiled
unchanged from src/main.c and tests/dump_model_stages.c: bit for bit."""
import ctypes as C

import numpy as np
import pytest

from oracle import Oracle, Reference

pytestmark = pytest.mark.skipif(not Reference.available(), reason="reference library not built")

# (src_h, src_w, out_h, out_w): down / up / identity / odd / one-pixel edges
SHAPES = [(480, 640, 640, 640), (720, 1280, 640, 640), (37, 100, 96, 64), (640, 640, 640, 640), (1, 1, 32, 32),
          (7, 5, 1, 1), (5, 9, 3, 1), (333, 211, 160, 224)]


def _img(sh, sw, seed):
    return np.random.default_rng(seed).integers(0, 256, size=(sh, sw, 3), dtype=np.uint8)


@pytest.mark.parametrize("sh,sw,oh,ow", SHAPES)
def test_align_corners_resize_and_scale(sh, sw, oh, ow):
    src = _img(sh, sw, sh * 7 + sw)
    R = Reference.lib()
    ref = np.zeros((oh, ow, 3), np.uint8)
    R.ref_resize_rgb_bilinear(src.ctypes.data, sw, sh, ref.ctypes.data, ow, oh)
    ref_nchw = np.zeros((3, oh, ow), np.float32)
    R.ref_preprocess(ref_nchw.ctypes.data, ref.ctypes.data, ow, oh)
    got = Oracle.preprocess(src[None], oh, ow, mode=0)[0]
    assert np.array_equal(got.view(np.uint32), ref_nchw.view(np.uint32))


@pytest.mark.parametrize("sh,sw,oh,ow", SHAPES)
def test_half_pixel_resize(sh, sw, oh, ow, tmp_path):
    """load_rgb_resized decodes a file: the image goes through the reference's
    own BMP writer (lossless) first."""
    src = _img(sh, sw, sh * 11 + sw)
    R = Reference.lib()
    path = str(tmp_path / "img.bmp")
    assert R.visualize_write_bmp_rgb24(path.encode(), src.ctypes.data, sw, sh) == 0
    ptr = R.ref_load_rgb_resized(path.encode(), ow, oh)
    assert ptr
    try:
        ref = np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_uint8)), shape=(oh * ow * 3,)).copy()
    finally:
        R.ref_free(ptr)
    ref_nchw = np.zeros((3, oh, ow), np.float32)
    R.ref_preprocess(ref_nchw.ctypes.data, ref.ctypes.data, ow, oh)
    got = Oracle.preprocess(src[None], oh, ow, mode=1)[0]
    assert np.array_equal(got.view(np.uint32), ref_nchw.view(np.uint32))


def _rows(n, seed, thr):
    rng = np.random.default_rng(seed)
    r = rng.standard_normal((n, 6)).astype(np.float32) * 100
    r[:, 4] = rng.choice([thr, np.nextafter(np.float32(thr), np.float32(1)), 0.0, 0.9, -1.0, np.nan], size=n)
    r[:, 5] = rng.integers(0, 80, n).astype(np.float32)
    return r


@pytest.mark.parametrize("n,cap", [(300, 100), (300, 5), (40, 100), (0, 10), (33, 0)])
def test_decode_detections_oracle_vs_reference(n, cap):
    """Our decode restatement against the reference's decode_detections
    (detection.c:3-34), including scores equal to the threshold and NaN."""
    import yolo_b200 as yb

    thr = np.float32(0.25)
    rows = _rows(n, n + cap, thr)
    want, cnt = Oracle.decode_detections(rows, thr, cap)
    R = Reference.lib()

    class Res(C.Structure):
        _fields_ = [("detections", C.c_void_p), ("count", C.c_int), ("capacity", C.c_int)]

    buf = np.zeros(max(cap, 1), dtype=Oracle.DET_DTYPE)
    res = Res(buf.ctypes.data, 0, cap)
    src = np.ascontiguousarray(rows.reshape(1, n, 6, 1)) if n else np.zeros((1, 0, 6, 1), np.float32)
    t = yb.Tensor()
    t.data = src.ctypes.data_as(C.POINTER(C.c_float))
    for i, d in enumerate((1, n, 6, 1)):
        t.dims[i] = d
    R.decode_detections.argtypes = [C.c_void_p, C.c_void_p, C.c_float]
    assert R.decode_detections(C.byref(res), C.byref(t), thr) == 0
    assert res.count == cnt
    assert buf[:cnt].tobytes() == want[:cnt].tobytes()
