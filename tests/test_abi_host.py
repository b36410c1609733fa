"""CPU-only checks of the C ABI: the library loads, exports every function
that include/*.h declares, and the host-side entry points (no device work)
behave like the reference's (tests/test_core.c of phucb2/yolo-baremetal)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def _declared_functions():
    names = set()
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"typedef[^;]*;", "", text)  # function-pointer typedefs are not exports
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\([^;{]*\)\s*;", text, re.M):
            if m.group(1) not in ("typedef", "if", "return"):
                names.add(m.group(1))
    return names


def test_library_exports_every_declared_function():
    import yolo_b200 as yb

    declared = _declared_functions()
    assert len(declared) >= 50
    lib = yb.lib()
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    listed = {s for syms in yb.EXPORTS.values() for s in syms}
    assert declared == listed, sorted(declared ^ listed)


def test_tensor_lifecycle():
    import yolo_b200 as yb

    L = yb.lib()
    t = yb.Tensor()
    assert L.tensor_allocate(C.byref(t), 1, 3, 4, 5) == yb.SUCCESS
    assert list(t.dims) == [1, 3, 4, 5] and list(t.stride) == [60, 20, 5, 1] and t.is_owner
    assert L.tensor_fill(C.byref(t), C.c_float(2.5)) == yb.SUCCESS
    u = yb.Tensor()
    L.tensor_allocate(C.byref(u), 1, 3, 4, 5)
    assert L.tensor_copy(C.byref(u), C.byref(t)) == yb.SUCCESS
    assert np.all(np.ctypeslib.as_array(u.data, shape=(60,)) == 2.5)
    v = yb.Tensor()
    L.tensor_allocate(C.byref(v), 1, 3, 4, 6)
    assert L.tensor_copy(C.byref(v), C.byref(t)) == yb.ERROR_INVALID_DIMS
    assert L.tensor_copy(None, C.byref(t)) == yb.ERROR_NULL_POINTER
    for x in (t, u, v):
        assert L.tensor_free(C.byref(x)) == yb.SUCCESS


def test_named_tensor_roundtrip_and_truncation(tmp_path):
    import yolo_b200 as yb

    L = yb.lib()
    libc = C.CDLL(None)
    libc.fopen.restype = C.c_void_p
    libc.fopen.argtypes = [C.c_char_p, C.c_char_p]
    libc.fclose.argtypes = [C.c_void_p]
    L.save_named_tensor.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(yb.Tensor)]
    L.load_named_tensor.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(yb.Tensor)]
    a = np.arange(24, dtype=np.float32).reshape(1, 2, 3, 4)
    path = str(tmp_path / "t.bin").encode()
    f = libc.fopen(path, b"wb")
    assert L.save_named_tensor(f, b"stage_01_buf0", C.byref(yb.tensor_view(a))) == yb.SUCCESS
    libc.fclose(f)
    name = C.create_string_buffer(128)
    t = yb.Tensor()
    f = libc.fopen(path, b"rb")
    assert L.load_named_tensor(f, name, C.byref(t)) == yb.SUCCESS
    assert name.value == b"stage_01_buf0" and list(t.dims) == [1, 2, 3, 4]
    assert np.array_equal(np.ctypeslib.as_array(t.data, shape=(24,)), a.reshape(-1))
    assert L.load_named_tensor(f, name, C.byref(yb.Tensor())) == yb.ERROR_FILE_NOT_FOUND  # end of file
    libc.fclose(f)
    L.tensor_free(C.byref(t))
    data = open(path, "rb").read()
    open(path, "wb").write(data[:-8])  # truncated data block
    f = libc.fopen(path, b"rb")
    assert L.load_named_tensor(f, name, C.byref(yb.Tensor())) == yb.ERROR_INVALID_FORMAT
    libc.fclose(f)


def test_fold_bn_known_answer():
    """test_core.c:86-110: w=2, b=1, gamma=1, beta=0, mean=0, var=1."""
    import yolo_b200 as yb

    L = yb.lib()
    arrs = [np.array([v], dtype=np.float32) for v in (2.0, 1.0, 1.0, 0.0, 0.0, 1.0)]
    ts = [yb.tensor_view(a) for a in arrs]
    L.fold_bn(*[C.byref(t) for t in ts])
    scale = np.float32(1.0) / np.sqrt(np.float32(1.0) + np.float32(1e-5))
    assert abs(arrs[0][0] - 2.0 * scale) < 1e-6 and abs(arrs[1][0] - scale) < 1e-6


def test_decode_detections_known_answer():
    """test_core.c:467-489."""
    import yolo_b200 as yb

    class Det(C.Structure):
        _fields_ = [("x1", C.c_float), ("y1", C.c_float), ("x2", C.c_float), ("y2", C.c_float),
                    ("score", C.c_float), ("class_id", C.c_int)]

    class Res(C.Structure):
        _fields_ = [("detections", C.POINTER(Det)), ("count", C.c_int), ("capacity", C.c_int)]

    head = np.zeros((1, 2, 6, 1), dtype=np.float32)
    head[0, 0, :, 0] = [256, 192, 384, 288, 0.95, 3]
    dets = (Det * 2)()
    res = Res(dets, 0, 2)
    assert yb.lib().decode_detections(C.byref(res), C.byref(yb.tensor_view(head)), C.c_float(0.5)) == yb.SUCCESS
    assert res.count == 1 and dets[0].class_id == 3 and abs(dets[0].x1 - 256) < 1 and abs(dets[0].y1 - 192) < 1


def test_profile_step_names():
    import yolo_b200 as yb

    L = yb.lib()
    assert L.model_forward_profile_step_name(0) == b"conv model.0 /2 + SiLU"
    assert L.model_forward_profile_step_name(23).startswith(b"Detect one2one")
    assert L.model_forward_profile_step_name(25) == b"?"


def test_weights_bin_roundtrip(tmp_path):
    import yb_weights as yw

    sd = yw.random_state("n", 3)
    p = str(tmp_path / "w.bin")
    yw.write_bin(p, sd, nc=80)
    nc, back = yw.read_bin(p)
    assert nc == 80 and list(back) == sorted(sd) and all(np.array_equal(back[k], sd[k]) for k in sd)
    # unfused Conv+BN records for every conv, plain Conv2d heads, both Detect branches
    assert "model.0.bn.running_var" in back and "model.23.one2one_cv3.0.2.bias" in back


def test_oracle_fold_matches_numpy(weights_n0):
    """The oracle's BN fold (utils.c:81-106 arithmetic) on the generated weights."""
    import yb_weights as yw
    from oracle import Oracle

    _, raw = yw.read_bin(weights_n0)
    o = Oracle(weights_n0)
    p = "model.2.m.0.cv1"
    g, b, mu, var = (raw[f"{p}.bn.{k}"] for k in ("weight", "bias", "running_mean", "running_var"))
    scale = (g / np.sqrt(var + np.float32(1e-5))).astype(np.float32)
    w = raw[f"{p}.conv.weight"] * scale[:, None, None, None]
    bias = (np.float32(0) - mu) * scale + b
    assert np.allclose(o.get(f"{p}.conv.weight"), w.reshape(-1), rtol=1e-6, atol=1e-7)
    assert np.allclose(o.get(f"{p}.conv.bias"), bias, rtol=1e-6, atol=1e-7)
    assert o.get(f"{p}.bn.weight") is None


def test_no_device_fails_cleanly():
    """Without a usable GPU the device entry points return a status, never crash."""
    from conftest import gpu_present
    import yolo_b200 as yb

    if gpu_present():
        pytest.skip("a GPU is present")
    ctx = C.c_void_p()
    st = yb.lib().yb_cuda_init(0, C.byref(ctx))
    assert st != yb.SUCCESS and not ctx.value
    assert yb.last_error()


def test_fold_bn_matches_oracle():
    """fold_bn (utils.c:81-106 arithmetic) on the reference's raw Conv+BN
    records gives the oracle's folded weights and bias bit for bit."""
    import yolo_b200 as yb
    from conftest import golden
    from oracle import Oracle

    r = golden("c3k2_test.bin")
    o = Oracle(nc=80)
    for k, v in r.items():
        if k not in ("input", "output"):
            o.add(f"X.{k}", v if v.ndim else v.reshape(1))
    o.fold()
    for prefix in ("cv1", "m.0.m.1.cv2", "m.1.cv3"):
        w = np.array(r[f"{prefix}.conv.weight"], dtype=np.float32, copy=True)
        b = np.zeros(w.shape[0], dtype=np.float32)
        tv = lambda a: C.byref(yb.tensor_view(a))  # noqa: E731
        yb.lib().fold_bn(tv(w), tv(b), tv(r[f"{prefix}.bn.weight"]), tv(r[f"{prefix}.bn.bias"]),
                         tv(r[f"{prefix}.bn.running_mean"]), tv(r[f"{prefix}.bn.running_var"]))
        assert np.array_equal(w.reshape(-1), o.get(f"X.{prefix}.conv.weight")), prefix
        assert np.array_equal(b, o.get(f"X.{prefix}.conv.bias")), prefix


def test_tensor_view_keeps_its_array_alive():
    """A tensor_t view over a temporary array stays valid after the caller drops it."""
    import gc
    import weakref

    import yolo_b200 as yb

    a = np.arange(12, dtype=np.float32)
    wr = weakref.ref(a)
    t = yb.tensor_view(a)
    del a
    gc.collect()
    assert wr() is not None
    assert np.ctypeslib.as_array(t.data, shape=(12,))[11] == 11.0


def test_postprocess_topk_limit_is_reported():
    """detect_postprocess_from_pred keeps at most 1024 rows (the device top-k
    limit; the reference has none): a larger min(max_det, N, rows) is refused
    with ERROR_INVALID_DIMS before any device work, with the limit named."""
    import yolo_b200 as yb

    L = yb.lib()
    N, nc, rows = 2000, 3, 1500
    pred = np.zeros((N, 4 + nc), np.float32)
    out = yb.tensor_view(np.zeros((1, rows, 6, 1), np.float32))
    st = L.detect_postprocess_from_pred(pred.ctypes.data_as(C.POINTER(C.c_float)), N, nc, 1500, C.byref(out))
    assert st == yb.ERROR_INVALID_DIMS
    assert "1024" in yb.last_error()
