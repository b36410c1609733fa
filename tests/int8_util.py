"""Shared helpers for the INT8 convolution tests: seeded layer data, the
library quantiser and the CPU oracle (test infrastructure) through ctypes."""
import ctypes as C

import numpy as np


def orc_lib():
    from oracle import Oracle

    L = Oracle.lib()
    if not getattr(L, "_i8_bound", False):
        L.orc_i8_quantize_conv.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                           C.c_float, C.c_float, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_void_p, C.c_void_p]
        L.orc_i8_conv.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                  C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.orc_i8_rshift_rne.argtypes = [C.c_int64, C.c_int]
        L.orc_i8_rshift_rne.restype = C.c_int64
        L._i8_bound = True
    return L


def ptr(a):
    return a.ctypes.data if a is not None else None


def make_layer(ci, co, k, H, W, B=1, seed=0, act=True, bias=True):
    """Seeded int8 input (NHWC), fp32 Kaiming weights and bias, and per-tensor
    scales: s_in fixed, s_pre / s_out from the float output range of the
    dequantised input (about 1 % of outputs saturate)."""
    import torch

    rng = np.random.default_rng(seed)
    s_in = np.float32(0.02)
    xq = rng.integers(-127, 128, size=(B, H, W, ci), dtype=np.int8)
    w = (rng.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
    b = (rng.standard_normal(co) * 0.1).astype(np.float32) if bias else None
    pad = (k - 1) // 2
    xf = torch.from_numpy(xq.astype(np.float32) * s_in).permute(0, 3, 1, 2)
    yf = torch.nn.functional.conv2d(xf, torch.from_numpy(w), torch.from_numpy(b) if bias else None, padding=pad)
    s_pre = np.float32(float(yf.abs().quantile(0.99)) / 127.0) if yf.numel() < 2**24 else np.float32(
        float(yf.abs().max()) * 0.7 / 127.0)
    silu = yf * torch.sigmoid(yf)
    s_out = np.float32(float(silu.abs().max()) / 127.0) if act else s_pre
    return dict(xq=xq, w=w, b=b, s_in=s_in, s_pre=s_pre, s_out=s_out, act=act, pad=pad)


def quantize_lib(lyr):
    import yolo_b200 as yb

    co, ci, k = lyr["w"].shape[0], lyr["w"].shape[1], lyr["w"].shape[2]
    q = dict(wq=np.zeros((co, ci, k, k), np.int8), bq=np.zeros(co, np.int32), mult=np.zeros(co, np.int32),
             shift=np.zeros(co, np.int32), lut=np.zeros(256, np.int8) if lyr["act"] else None)
    st = yb.lib().yb_int8_quantize_conv(ptr(lyr["w"]), ptr(lyr["b"]), co, ci, k, k, lyr["s_in"], lyr["s_pre"],
                                        lyr["s_out"], int(lyr["act"]), ptr(q["wq"]), ptr(q["bq"]), ptr(q["mult"]),
                                        ptr(q["shift"]), ptr(q["lut"]))
    yb.check(st, "yb_int8_quantize_conv")
    return q


def quantize_oracle(lyr):
    co, ci, k = lyr["w"].shape[0], lyr["w"].shape[1], lyr["w"].shape[2]
    q = dict(wq=np.zeros((co, ci, k, k), np.int8), bq=np.zeros(co, np.int32), mult=np.zeros(co, np.int32),
             shift=np.zeros(co, np.int32), lut=np.zeros(256, np.int8) if lyr["act"] else None)
    assert orc_lib().orc_i8_quantize_conv(ptr(lyr["w"]), ptr(lyr["b"]), co, ci, k, k, lyr["s_in"], lyr["s_pre"],
                                          lyr["s_out"], int(lyr["act"]), ptr(q["wq"]), ptr(q["bq"]), ptr(q["mult"]),
                                          ptr(q["shift"]), ptr(q["lut"])) == 0
    return q


def conv_oracle(xq, q, k, stride, pad):
    B, H, W, ci = xq.shape
    co = q["wq"].shape[0]
    Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    y = np.zeros((B, Ho, Wo, co), np.int8)
    x = np.ascontiguousarray(xq)
    assert orc_lib().orc_i8_conv(ptr(x), B, H, W, ci, ptr(q["wq"]), ptr(q["bq"]), ptr(q["mult"]), ptr(q["shift"]),
                                 ptr(q["lut"]), co, k, k, stride, pad, ptr(y)) == 0
    return y
