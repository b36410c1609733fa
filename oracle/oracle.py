"""ctypes access to the CPU oracle -- TEST INFRASTRUCTURE ONLY.

`Oracle` wraps liboracle.so (our C restatement of the reference forward, see
yolo_oracle.c) and `Reference` wraps _ref/libyolo_ref.so (the reference's own
sources compiled by oracle/Makefile plus ref_harness.c).  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use this module; the
product never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from collections import OrderedDict

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libyolo_ref.so")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
STAGE_CB = C.CFUNCTYPE(None, C.c_void_p, C.c_char_p, C.POINTER(C.c_float), C.c_int, C.c_int, C.c_int, C.c_int)


def build() -> None:
    """Builds liboracle.so (and _ref when the reference sources are present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _collector(store: "OrderedDict[str, np.ndarray]"):
    def cb(_user, name, data, n, c, h, w):
        cnt = n * c * h * w
        arr = np.ctypeslib.as_array(data, shape=(cnt,)).copy().reshape(n, c, h, w)
        store[name.decode()] = arr

    return STAGE_CB(cb)


I8_STAGE_CB = C.CFUNCTYPE(None, C.c_void_p, C.c_char_p, C.POINTER(C.c_int8), C.POINTER(C.c_float), C.c_int,
                          C.c_int, C.c_int)


class Oracle:
    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            if not os.path.exists(ORACLE_SO):
                build()
            lib = C.CDLL(ORACLE_SO)
            lib.orc_new.restype = C.c_void_p
            lib.orc_new.argtypes = [C.c_int]
            lib.orc_load.restype = C.c_void_p
            lib.orc_load.argtypes = [C.c_char_p]
            lib.orc_free.argtypes = [C.c_void_p]
            lib.orc_add.argtypes = [C.c_void_p, C.c_char_p, C.POINTER(C.c_int), _f32p]
            lib.orc_fold.argtypes = [C.c_void_p]
            lib.orc_get.restype = C.c_long
            lib.orc_get.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_long]
            lib.orc_forward.argtypes = [C.c_void_p, _f32p, C.c_int, C.c_int, C.c_int, _f32p, C.c_void_p, C.c_void_p,
                                        STAGE_CB, C.c_void_p]
            lib.orc_anchors.argtypes = [C.c_int, C.c_int]
            lib.orc_postprocess.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
            lib.orc_conv_block.argtypes = [C.c_void_p, C.c_char_p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                           C.c_int, _f32p]
            lib.orc_c3k2.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, _f32p,
                                     C.c_int]
            lib.orc_c3k2_c3k.argtypes = [C.c_void_p, C.c_char_p, _f32p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int]
            lib.orc_sppf.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int, C.c_int,
                                     C.c_int, _f32p, C.c_int]
            lib.orc_c2psa.argtypes = [C.c_void_p, C.c_char_p, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int]
            lib.orc_c3.argtypes = [C.c_void_p, C.c_char_p, C.c_int, _f32p, C.c_int, C.c_int, C.c_int, _f32p, C.c_int]
            lib.orc_stats_enable.argtypes = [C.c_void_p, C.c_int]
            lib.orc_stats_count.argtypes = [C.c_void_p]
            lib.orc_stats_entry.argtypes = [C.c_void_p, C.c_int, C.c_char_p, C.c_int, C.POINTER(C.c_float)]
            lib.orc_nc.argtypes = [C.c_void_p]
            lib.orc_i8_forward.argtypes = [C.c_void_p, C.POINTER(C.c_char_p), C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                           C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, I8_STAGE_CB,
                                           C.c_void_p]
            lib.orc_psablock.argtypes = [C.c_void_p, C.c_char_p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
            lib.orc_dwconv.argtypes = [C.c_void_p, C.c_char_p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
            for fn in (lib.orc_resize_align_corners, lib.orc_resize_half_pixel):
                fn.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int]
            lib.orc_rgb_to_nchw.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
            lib.orc_decode_detections.argtypes = [_f32p, C.c_int, C.c_int, C.c_float, C.c_int, C.c_void_p]
            cls._lib = lib
        return cls._lib

    def __init__(self, path: str | None = None, nc: int = 80):
        lib = self.lib()
        self.h = lib.orc_load(path.encode()) if path else lib.orc_new(nc)
        if not self.h:
            raise RuntimeError(f"oracle could not load {path}")

    def __del__(self):
        if getattr(self, "h", None):
            self.lib().orc_free(self.h)
            self.h = None

    def add(self, name: str, arr: np.ndarray) -> None:
        a = np.ascontiguousarray(arr, dtype=np.float32)
        dims = list(a.shape) + [1] * (4 - a.ndim)
        if a.ndim == 1:
            dims = [a.shape[0], 1, 1, 1]
        d = (C.c_int * 4)(*dims)
        if self.lib().orc_add(self.h, name.encode(), d, a.reshape(-1)) != 0:
            raise RuntimeError("orc_add failed")

    def fold(self) -> None:
        self.lib().orc_fold(self.h)

    def get(self, name: str) -> np.ndarray | None:
        n = self.lib().orc_get(self.h, name.encode(), None, 0)
        if n < 0:
            return None
        out = np.empty(n, dtype=np.float32)
        self.lib().orc_get(self.h, name.encode(), out.ctypes.data, n)
        return out

    def forward(self, img: np.ndarray, max_det: int = 300, stages: bool = False):
        """img [1,3,H,W] -> dict(dets [max_det,6], logits [N,nc], boxes [N,4], stages)."""
        x = np.ascontiguousarray(img, dtype=np.float32).reshape(-1)
        H, W = img.shape[-2], img.shape[-1]
        N = self.lib().orc_anchors(H, W)
        dets = np.zeros(max_det * 6, dtype=np.float32)
        logits = np.zeros(N * 80, dtype=np.float32)
        boxes = np.zeros(N * 4, dtype=np.float32)
        store: "OrderedDict[str, np.ndarray]" = OrderedDict()
        cb = _collector(store) if stages else STAGE_CB()
        st = self.lib().orc_forward(self.h, x, H, W, max_det, dets, logits.ctypes.data, boxes.ctypes.data, cb, None)
        if st != 0:
            raise RuntimeError(f"orc_forward status {st}")
        return {"dets": dets.reshape(max_det, 6), "logits": logits.reshape(N, -1), "boxes": boxes.reshape(N, 4),
                "stages": store}

    # ---------------------------------------------------------------- INT8
    def calibrate(self, images) -> "OrderedDict[str, float]":
        """Scale table (name -> max|x| / 127, 1.0 for an all-zero tensor) from
        FP32 forwards of `images` ([n,3,H,W])."""
        L = self.lib()
        L.orc_stats_enable(self.h, 1)
        try:
            for img in images:
                self.forward(img[None])
            table: "OrderedDict[str, float]" = OrderedDict()
            name = C.create_string_buffer(128)
            v = C.c_float()
            for i in range(L.orc_stats_count(self.h)):
                L.orc_stats_entry(self.h, i, name, 128, C.byref(v))
                a = np.float32(v.value)
                table[name.value.decode()] = float(a / np.float32(127.0)) if a > 0 else 1.0
        finally:
            L.orc_stats_enable(self.h, 0)
        return table

    def forward_i8(self, img: np.ndarray, scales, max_det: int = 300, stages: bool = False):
        """INT8 forward of img [1,3,H,W] under the scale table `scales`:
        dict(dets, logits [N,nc], dist [N,4], stages {name: (int8 [C,H,W], scales [C])})."""
        L = self.lib()
        x = np.ascontiguousarray(img, dtype=np.float32).reshape(-1)
        H, W = img.shape[-2], img.shape[-1]
        N = L.orc_anchors(H, W)
        nc = L.orc_nc(self.h)
        names = (C.c_char_p * len(scales))(*[k.encode() for k in scales])
        vals = np.array(list(scales.values()), dtype=np.float32)
        dets = np.zeros(max_det * 6, np.float32)
        logits = np.zeros(N * nc, np.float32)
        dist = np.zeros(N * 4, np.float32)
        store: "OrderedDict[str, tuple]" = OrderedDict()

        def _cb(_u, name, data, sc, c, h, w):
            store[name.decode()] = (np.ctypeslib.as_array(data, shape=(c * h * w,)).copy().reshape(c, h, w),
                                    np.ctypeslib.as_array(sc, shape=(c,)).copy())

        cb = I8_STAGE_CB(_cb) if stages else I8_STAGE_CB()
        st = L.orc_i8_forward(self.h, names, vals.ctypes.data, len(vals), x.ctypes.data, H, W, max_det,
                              dets.ctypes.data, logits.ctypes.data, dist.ctypes.data, cb, None)
        if st != 0:
            raise RuntimeError(f"orc_i8_forward status {st}")
        return {"dets": dets.reshape(max_det, 6), "logits": logits.reshape(N, nc), "dist": dist.reshape(N, 4),
                "stages": store}

    @classmethod
    def postprocess(cls, pred: np.ndarray, nc: int, max_det: int, cap: int) -> np.ndarray:
        out = np.zeros(cap * 6, dtype=np.float32)
        p = np.ascontiguousarray(pred, dtype=np.float32).reshape(-1)
        n = p.size // (4 + nc)
        cls.lib().orc_postprocess(p if p.size else np.zeros(1, np.float32), n, nc, max_det, cap, out)
        return out.reshape(cap, 6)

    DET_DTYPE = np.dtype([("x1", np.float32), ("y1", np.float32), ("x2", np.float32), ("y2", np.float32),
                          ("score", np.float32), ("class_id", np.int32)])

    @classmethod
    def decode_detections(cls, rows: np.ndarray, threshold: float, capacity: int):
        """decode_detections for one image's [n, 6] rows: (structured array [capacity], count)."""
        r = np.ascontiguousarray(rows, dtype=np.float32)
        out = np.zeros(max(capacity, 1), dtype=cls.DET_DTYPE)
        n = cls.lib().orc_decode_detections(r.reshape(-1), r.shape[0], r.shape[1], threshold, capacity,
                                            out.ctypes.data)
        return out[:capacity], n

    @classmethod
    def preprocess(cls, rgb: np.ndarray, H: int, W: int, mode: int = 0) -> np.ndarray:
        """uint8 HWC RGB images [B, sh, sw, 3] -> fp32 NCHW [B, 3, H, W]: resize
        (mode 0: src/main.c resize_rgb_bilinear; mode 1: the pixel-centred
        resize of tests/dump_model_stages.c) then / 255."""
        L = cls.lib()
        rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
        B, sh, sw, _ = rgb.shape
        out = np.zeros((B, 3, H, W), np.float32)
        tmp = np.zeros((H, W, 3), np.uint8)
        fn = L.orc_resize_align_corners if mode == 0 else L.orc_resize_half_pixel
        for b in range(B):
            fn(rgb[b].ctypes.data, sw, sh, tmp.ctypes.data, W, H)
            L.orc_rgb_to_nchw(tmp.ctypes.data, W, H, out[b].ctypes.data)
        return out


class Reference:
    """The reference implementation compiled from its own sources."""

    _lib = None

    @classmethod
    def available(cls) -> bool:
        return os.path.exists(REF_SO)

    @classmethod
    def lib(cls):
        if cls._lib is None:
            lib = C.CDLL(REF_SO)
            lib.ref_forward.argtypes = [C.c_char_p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p, C.c_char_p,
                                        C.c_void_p]
            lib.ref_time_forwards.restype = C.c_double
            lib.ref_time_forwards.argtypes = [C.c_char_p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int]
            lib.ref_postprocess.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_int, _f32p]
            lib.ref_resize_rgb_bilinear.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int]
            lib.ref_preprocess.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int]
            lib.ref_load_rgb_resized.restype = C.c_void_p
            lib.ref_load_rgb_resized.argtypes = [C.c_char_p, C.c_int, C.c_int]
            lib.ref_free.argtypes = [C.c_void_p]
            lib.visualize_write_bmp_rgb24.argtypes = [C.c_char_p, C.c_void_p, C.c_int, C.c_int]
            cls._lib = lib
        return cls._lib

    @classmethod
    def forward(cls, weights: str, img: np.ndarray, width_mult: int = 1, max_det: int = 300,
                stage_path: str | None = None, logits: bool = True, nc: int = 80):
        H, W = img.shape[-2], img.shape[-1]
        x = np.ascontiguousarray(img, dtype=np.float32).reshape(-1)
        N = (H // 8) * (W // 8) + (H // 16) * (W // 16) + (H // 32) * (W // 32)
        dets = np.zeros(max_det * 6, dtype=np.float32)
        lg = np.zeros(N * nc, dtype=np.float32) if logits else None
        st = cls.lib().ref_forward(weights.encode(), x, H, W, width_mult, max_det, dets,
                                   stage_path.encode() if stage_path else None,
                                   lg.ctypes.data if lg is not None else None)
        if st != 0:
            raise RuntimeError(f"reference forward status {st}")
        return {"dets": dets.reshape(max_det, 6), "logits": lg.reshape(N, nc) if lg is not None else None}

    @classmethod
    def time_forwards(cls, weights: str, img: np.ndarray, reps: int, width_mult: int = 1) -> float:
        H, W = img.shape[-2], img.shape[-1]
        x = np.ascontiguousarray(img, dtype=np.float32).reshape(-1)
        t = cls.lib().ref_time_forwards(weights.encode(), x, H, W, width_mult, reps)
        if t < 0:
            raise RuntimeError(f"reference timing failed ({t})")
        return t

    @classmethod
    def postprocess(cls, pred: np.ndarray, nc: int, max_det: int, cap: int) -> np.ndarray:
        out = np.zeros(cap * 6, dtype=np.float32)
        p = np.ascontiguousarray(pred, dtype=np.float32).reshape(-1)
        n = p.size // (4 + nc)
        st = cls.lib().ref_postprocess(p if p.size else np.zeros(1, np.float32), n, nc, max_det, cap, out)
        if st != 0:
            raise RuntimeError(f"reference postprocess status {st}")
        return out.reshape(cap, 6)
