"""Python binding of libyolo_b200.so through its C ABI (ctypes).

The library is the product: sm_100a kernels behind the reference's host API
(include/{tensor,layers,model,detect,detection,utils}.h) and the yb_cuda_*
shim (include/yb_cuda.h).  This module only marshals numpy arrays into those
C calls; it never computes a result itself, and it raises when the library is
missing rather than falling back to anything else.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libyolo_b200.so")

# status_t (include/status.h)
STATUS = ["SUCCESS", "ERROR_NULL_POINTER", "ERROR_INVALID_DIMS", "ERROR_OUT_OF_MEMORY", "ERROR_NOT_IMPLEMENTED",
          "ERROR_FILE_NOT_FOUND", "ERROR_INVALID_FORMAT", "ERROR_DEVICE", "ERROR_TIMEOUT"]
SUCCESS, ERROR_NULL_POINTER, ERROR_INVALID_DIMS, ERROR_OUT_OF_MEMORY, ERROR_NOT_IMPLEMENTED, \
    ERROR_FILE_NOT_FOUND, ERROR_INVALID_FORMAT, ERROR_DEVICE, ERROR_TIMEOUT = range(9)

# Exported C symbols, grouped by the header that declares them.
EXPORTS = {
    "tensor.h": ["tensor_allocate", "tensor_free", "tensor_copy", "tensor_fill", "tensor_gemm", "malloc_aligned",
                 "free_aligned"],
    "layers.h": ["conv2d_forward", "silu_forward", "pool2d_max_forward", "upsample_nearest_forward", "concat_forward",
                 "conv_block_forward", "bottleneck_forward", "sppf_forward", "c3k2_forward", "c2psa_forward",
                 "psablock_forward", "dwconv3x3_same_forward", "c3_forward"],
    "model.h": ["model_forward_profile_reset", "model_forward_profile_step_name", "model_forward_profile_print_last",
                "model_forward_profile_print_aggregate", "model_create", "model_destroy", "model_forward",
                "model_forward_ex", "model_forward_batch", "model_load_weights", "model_get_weight"],
    "detect.h": ["detect_forward_one2one", "detect_postprocess_from_pred"],
    "detection.h": ["decode_detections"],
    "utils.h": ["timer_start", "timer_stop", "timer_elapsed_ms", "load_named_tensor", "save_named_tensor", "fold_bn"],
    "yb_cuda.h": ["yb_cuda_init", "yb_cuda_upload_weights", "yb_cuda_load_bin", "yb_cuda_forward",
                  "yb_cuda_set_int8", "yb_cuda_set_fusion", "yb_cuda_get_int8_stage", "yb_cuda_calibrate_int8",
                  "yb_cuda_int8_scale_entry", "yb_cuda_forward_rgb8", "yb_cuda_preprocess_rgb8",
                  "yb_cuda_forward_submit", "yb_cuda_forward_rgb8_submit", "yb_cuda_forward_wait",
                  "yb_cuda_get_detections", "yb_cuda_detections",
                  "yb_cuda_plan_io", "yb_cuda_forward_device", "yb_cuda_get_head", "yb_cuda_detect_topk_noalloc",
                  "yb_cuda_forward_sharded",
                  "yb_cuda_profile_ops", "yb_cuda_debug_inject_stall", "yb_cuda_destroy", "yb_cuda_last_error",
                  "yb_conv_create", "yb_conv_ci_pad", "yb_conv_run", "yb_conv_check", "yb_conv_destroy",
                  "yb_cuda_load_bin_device", "yb_cuda_save_prepared", "yb_cuda_load_prepared",
                  "yb_cuda_weight_image", "yb_conv_debug_withhold"],
    "yb_int8.h": ["yb_int8_quantize_conv", "yb_int8_conv_create", "yb_int8_conv_ci_pad", "yb_int8_conv_run",
                  "yb_int8_conv_check", "yb_int8_conv_destroy"],
}


# detection_t (include/detection.h)
DET_DTYPE = np.dtype([("x1", np.float32), ("y1", np.float32), ("x2", np.float32), ("y2", np.float32),
                      ("score", np.float32), ("class_id", np.int32)])


class YBError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str = ""):
        self.status = status
        name = STATUS[status] if 0 <= status < len(STATUS) else str(status)
        super().__init__(f"{where}: {name}" + (f" ({detail})" if detail else ""))


class Tensor(C.Structure):
    """tensor_t (include/tensor.h)."""

    _fields_ = [("data", C.POINTER(C.c_float)), ("dims", C.c_int * 4), ("stride", C.c_int * 4), ("is_owner", C.c_bool)]


class ConvParams(C.Structure):
    _fields_ = [("stride", C.c_int), ("padding", C.c_int), ("groups", C.c_int)]


class ModelT(C.Structure):
    """model_t (include/model.h)."""

    _fields_ = [("weights", C.c_void_p), ("num_weights", C.c_int), ("buffers", C.POINTER(Tensor)),
                ("num_buffers", C.c_int), ("input_w", C.c_int), ("input_h", C.c_int), ("num_classes", C.c_int)]


class Profile(C.Structure):
    _fields_ = [("ms_sum", C.c_double * 25), ("ms_last", C.c_double * 25), ("runs", C.c_uint)]


def build(jobs: int = 8) -> None:
    subprocess.run(["make", "-s", "-C", HERE, f"-j{jobs}"], check=True)


_lib = None


def lib() -> C.CDLL:
    """Loads libyolo_b200.so; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` (no fallback exists)")
        L = C.CDLL(LIB_PATH)
        L.yb_cuda_last_error.restype = C.c_char_p
        L.yb_cuda_init.argtypes = [C.c_int, C.POINTER(C.c_void_p)]
        L.yb_cuda_load_bin.argtypes = [C.c_void_p, C.c_char_p]
        L.yb_cuda_forward.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                      C.c_void_p, C.c_void_p, C.c_void_p]
        L.yb_cuda_plan_io.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p),
                                      C.POINTER(C.c_void_p)]
        L.yb_cuda_forward_device.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                             C.c_void_p]
        L.yb_cuda_get_head.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.yb_cuda_detect_topk_noalloc.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                                  C.c_void_p, C.c_void_p]
        L.yb_cuda_forward_sharded.argtypes = [C.POINTER(C.c_void_p), C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                              C.c_void_p, C.c_int, C.c_int]
        L.yb_cuda_debug_inject_stall.argtypes = [C.c_void_p, C.c_int]
        L.yb_cuda_profile_ops.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                          C.c_int, C.POINTER(C.c_int)]
        L.yb_cuda_destroy.argtypes = [C.c_void_p]
        L.yb_conv_create.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.POINTER(C.c_void_p)]
        L.yb_conv_ci_pad.argtypes = [C.c_void_p]
        L.yb_cuda_load_bin_device.argtypes = [C.c_void_p, C.c_char_p]
        L.yb_cuda_save_prepared.argtypes = [C.c_void_p, C.c_char_p]
        L.yb_cuda_load_prepared.argtypes = [C.c_void_p, C.c_char_p]
        L.yb_cuda_weight_image.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t,
                                           C.POINTER(C.c_size_t)]
        L.yb_conv_run.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.yb_conv_check.argtypes = [C.c_void_p]
        L.yb_conv_debug_withhold.argtypes = [C.c_void_p]
        L.yb_conv_destroy.argtypes = [C.c_void_p]
        L.yb_cuda_set_int8.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.yb_cuda_set_fusion.argtypes = [C.c_void_p, C.c_int]
        L.yb_cuda_get_detections.argtypes = [C.c_void_p, C.c_float, C.c_int, C.c_void_p, C.c_void_p]
        L.yb_cuda_detections.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_int, C.c_void_p, C.c_void_p,
                                         C.c_void_p]
        L.yb_cuda_forward_rgb8.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                           C.c_int, C.c_void_p, C.c_int]
        L.yb_cuda_preprocess_rgb8.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                              C.c_int, C.c_void_p]
        L.yb_cuda_forward_submit.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int,
                                             C.POINTER(C.c_longlong)]
        L.yb_cuda_forward_rgb8_submit.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                  C.c_int, C.c_void_p, C.c_int, C.POINTER(C.c_longlong)]
        L.yb_cuda_forward_wait.argtypes = [C.c_void_p, C.c_longlong]
        L.yb_cuda_calibrate_int8.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                             C.POINTER(C.c_int)]
        L.yb_cuda_int8_scale_entry.argtypes = [C.c_void_p, C.c_int, C.c_char_p, C.c_int, C.POINTER(C.c_float)]
        L.yb_cuda_get_int8_stage.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                             C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.yb_int8_quantize_conv.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                            C.c_float, C.c_float, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                            C.c_void_p, C.c_void_p]
        L.yb_int8_conv_create.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                          C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.POINTER(C.c_void_p)]
        L.yb_int8_conv_ci_pad.argtypes = [C.c_void_p]
        L.yb_int8_conv_run.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.yb_int8_conv_check.argtypes = [C.c_void_p]
        L.yb_int8_conv_destroy.argtypes = [C.c_void_p]
        L.model_forward_profile_step_name.restype = C.c_char_p
        L.model_get_weight.restype = C.POINTER(Tensor)
        _lib = L
    return _lib


def last_error() -> str:
    return lib().yb_cuda_last_error().decode()


def check(status: int, where: str) -> None:
    if status != SUCCESS:
        raise YBError(status, where, last_error())


def tensor_view(a: np.ndarray) -> Tensor:
    """Non-owning tensor_t over a C-contiguous float32 array (1-4 dims; dims padded with 1)."""
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    dims = list(a.shape) + [1] * (4 - a.ndim)
    if a.ndim == 1:
        dims = [a.shape[0], 1, 1, 1]
    t = Tensor()
    t.data = a.ctypes.data_as(C.POINTER(C.c_float))
    t.dims[:] = dims
    t.stride[:] = [dims[1] * dims[2] * dims[3], dims[2] * dims[3], dims[3], 1]
    t.is_owner = False
    t._array = a  # the view must keep its array alive: tensor_t holds only the raw pointer
    return t


class Model:
    """One device replica (yb_cuda_* context) on one GPU."""

    def __init__(self, weights: str, device: int = 0, prep: str = "host"):
        """prep: "host" (fold and pack on the host), "device" (fold, pack and
        quantise on the GPU) or "blob" (weights is a prepared-weight blob)."""
        L = lib()
        self.ctx = C.c_void_p()
        check(L.yb_cuda_init(device, C.byref(self.ctx)), "yb_cuda_init")
        load = {"host": L.yb_cuda_load_bin, "device": L.yb_cuda_load_bin_device, "blob": L.yb_cuda_load_prepared}[prep]
        check(load(self.ctx, weights.encode()), f"load ({prep})")
        self.device = device

    def save_prepared(self, path: str) -> None:
        check(lib().yb_cuda_save_prepared(self.ctx, path.encode()), "yb_cuda_save_prepared")

    def weight_image(self, name: str, kind: int, n_tile: int = 0) -> bytes:
        """Prepared weight image (kind 0 folded fp32 tensor, 1 packed FP32 conv, 2 packed INT8 conv)."""
        n = C.c_size_t()
        check(lib().yb_cuda_weight_image(self.ctx, name.encode(), kind, n_tile, None, 0, C.byref(n)),
              "yb_cuda_weight_image")
        buf = C.create_string_buffer(n.value)
        check(lib().yb_cuda_weight_image(self.ctx, name.encode(), kind, n_tile, buf, n.value, C.byref(n)),
              "yb_cuda_weight_image")
        return buf.raw[: n.value]

    def close(self) -> None:
        if self.ctx:
            lib().yb_cuda_destroy(self.ctx)
            self.ctx = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, images: np.ndarray, max_det: int = 300, profile: bool = False, stages: bool = False):
        """images [B,3,H,W] float32 -> dets [B,max_det,6] (and optional per-step ms / stage dict)."""
        x = np.ascontiguousarray(images, dtype=np.float32)
        B, _, H, W = x.shape
        dets = np.zeros((B, max_det, 6), dtype=np.float32)
        ms = (C.c_double * 25)() if profile else None
        store = {}
        cb = None
        if stages:
            CB = C.CFUNCTYPE(None, C.c_void_p, C.c_char_p, C.POINTER(C.c_float), C.c_int, C.c_int, C.c_int, C.c_int)

            def _cb(_u, name, data, n, c, h, w):
                store[name.decode()] = np.ctypeslib.as_array(data, shape=(n * c * h * w,)).copy().reshape(n, c, h, w)

            cb = CB(_cb)
        check(lib().yb_cuda_forward(self.ctx, x.ctypes.data, B, H, W, dets.ctypes.data, max_det,
                                    C.cast(cb, C.c_void_p) if cb else None, None, ms), "yb_cuda_forward")
        out = {"dets": dets}
        if profile:
            out["step_ms"] = list(ms)
        if stages:
            out["stages"] = store
        return out

    def set_int8(self, scales=None) -> None:
        """INT8 mode under a scale table {tensor name: scale}; None or {} returns to FP32."""
        scales = dict(scales or {})
        n = len(scales)
        names = (C.c_char_p * max(n, 1))(*[k.encode() for k in scales])
        vals = np.ascontiguousarray(list(scales.values()) or [0.0], dtype=np.float32)
        check(lib().yb_cuda_set_int8(self.ctx, names, vals.ctypes.data, n), "yb_cuda_set_int8")

    def set_fusion(self, enable: bool) -> None:
        """Fused Bottleneck launches on (default) or off; results are bit-identical."""
        check(lib().yb_cuda_set_fusion(self.ctx, 1 if enable else 0), "yb_cuda_set_fusion")

    def calibrate_int8(self, images: np.ndarray, apply: bool = True) -> dict:
        """Device calibration from FP32 forwards of images [n,3,H,W]: {name: scale}; apply switches to INT8."""
        x = np.ascontiguousarray(images, dtype=np.float32)
        n = C.c_int()
        check(lib().yb_cuda_calibrate_int8(self.ctx, x.ctypes.data, x.shape[0], x.shape[2], x.shape[3],
                                           1 if apply else 0, C.byref(n)), "yb_cuda_calibrate_int8")
        out = {}
        name = C.create_string_buffer(256)
        v = C.c_float()
        for i in range(n.value):
            check(lib().yb_cuda_int8_scale_entry(self.ctx, i, name, 256, C.byref(v)), "yb_cuda_int8_scale_entry")
            out[name.value.decode()] = float(v.value)
        return out

    def int8_stage(self, idx: int, image: int = 0):
        """(int8 [C,H,W], per-channel scales [C]) of stage tensor idx (0..22) of the last INT8 forward."""
        c, h, w = C.c_int(), C.c_int(), C.c_int()
        check(lib().yb_cuda_get_int8_stage(self.ctx, idx, image, None, None, C.byref(c), C.byref(h), C.byref(w)),
              "yb_cuda_get_int8_stage")
        q = np.zeros((c.value, h.value, w.value), dtype=np.int8)
        cs = np.zeros(c.value, dtype=np.float32)
        check(lib().yb_cuda_get_int8_stage(self.ctx, idx, image, q.ctypes.data, cs.ctypes.data, None, None, None),
              "yb_cuda_get_int8_stage")
        return q, cs

    def forward_rgb8(self, rgb: np.ndarray, H: int = 640, W: int = 640, resize: int = 0, max_det: int = 300):
        """uint8 HWC RGB images [B, sh, sw, 3] -> dets [B, max_det, 6], preprocessed on the device."""
        x = np.ascontiguousarray(rgb, dtype=np.uint8)
        B, sh, sw, _ = x.shape
        dets = np.zeros((B, max_det, 6), dtype=np.float32)
        check(lib().yb_cuda_forward_rgb8(self.ctx, x.ctypes.data, B, sh, sw, resize, H, W, dets.ctypes.data, max_det),
              "yb_cuda_forward_rgb8")
        return dets

    def submit(self, x_ptr: int, B: int, H: int, W: int, out_ptr: int, max_det: int = 300) -> int:
        """Streaming forward: queues one batch (host pointers to [B,3,H,W] fp32 and [B,max_det,6] fp32, pinned
        for overlap, valid until wait) and returns its ticket."""
        t = C.c_longlong()
        check(lib().yb_cuda_forward_submit(self.ctx, x_ptr, B, H, W, out_ptr, max_det, C.byref(t)),
              "yb_cuda_forward_submit")
        return t.value

    def submit_rgb8(self, rgb_ptr: int, B: int, sh: int, sw: int, out_ptr: int, H: int = 640, W: int = 640,
                    resize: int = 0, max_det: int = 300) -> int:
        """Streaming forward from uint8 HWC frames [B, sh, sw, 3] (host pointer); returns the ticket."""
        t = C.c_longlong()
        check(lib().yb_cuda_forward_rgb8_submit(self.ctx, rgb_ptr, B, sh, sw, resize, H, W, out_ptr, max_det,
                                                C.byref(t)), "yb_cuda_forward_rgb8_submit")
        return t.value

    def wait(self, ticket: int) -> None:
        check(lib().yb_cuda_forward_wait(self.ctx, ticket), "yb_cuda_forward_wait")

    def detections(self, batch: int, threshold: float = 0.25, capacity: int = 100):
        """Detection lists of the last forward: (structured array [B, capacity], counts [B])."""
        out = np.zeros((batch, capacity), dtype=DET_DTYPE)
        counts = np.zeros(batch, dtype=np.int32)
        check(lib().yb_cuda_get_detections(self.ctx, threshold, capacity, out.ctypes.data, counts.ctypes.data),
              "yb_cuda_get_detections")
        return out, counts

    def head(self, batch: int):
        """(logits [B,N,nc], boxes [B,N,4]) of the last forward."""
        n = C.c_int()
        nc = C.c_int()
        check(lib().yb_cuda_get_head(self.ctx, None, None, C.byref(n), C.byref(nc)), "yb_cuda_get_head")
        logits = np.zeros((batch, n.value, nc.value), dtype=np.float32)
        boxes = np.zeros((batch, n.value, 4), dtype=np.float32)
        check(lib().yb_cuda_get_head(self.ctx, logits.ctypes.data, boxes.ctypes.data, None, None), "yb_cuda_get_head")
        return logits, boxes

    def plan_io(self, B: int, H: int, W: int, max_det: int = 300):
        d_in = C.c_void_p()
        d_out = C.c_void_p()
        check(lib().yb_cuda_plan_io(self.ctx, B, H, W, max_det, C.byref(d_in), C.byref(d_out)), "yb_cuda_plan_io")
        return d_in.value, d_out.value

    def forward_device(self, d_in: int, d_out: int, B: int, H: int, W: int, max_det: int = 300, stream: int = 0):
        check(lib().yb_cuda_forward_device(self.ctx, d_in, B, H, W, d_out, max_det, stream or None),
              "yb_cuda_forward_device")


def forward_sharded(models, images: np.ndarray, max_det: int = 300, timeout_ms: int = 0):
    x = np.ascontiguousarray(images, dtype=np.float32)
    B, _, H, W = x.shape
    dets = np.zeros((B, max_det, 6), dtype=np.float32)
    arr = (C.c_void_p * len(models))(*[m.ctx.value for m in models])
    st = lib().yb_cuda_forward_sharded(arr, len(models), x.ctypes.data, B, H, W, dets.ctypes.data, max_det,
                                       timeout_ms)
    return st, dets
