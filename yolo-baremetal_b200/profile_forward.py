"""Runs YOLO26 forwards for profiling: the command ncu wraps.

    python yolo-baremetal_b200/profile_forward.py [--batch 32] [--hw 640] [--width n] [--int8] [--ops]

Builds seeded random-init weights, runs one forward of `batch` seeded images
(plan build: one eager validation pass, then the captured graph), and with
--ops prints every launch of the plan with its device time (CUDA events),
algorithmic bytes and FLOPs (yb_cuda_profile_ops).  Under ncu, launch i of
conv_tc_kernel in the validation pass is the i-th convolution of the graph:
0 model.1, 1 model.2.cv1, 2 model.2.m.0.cv1, 3 model.2.m.0.cv2, 4 model.2.cv2, ...
With --int8 the forward is INT8, after a device calibration over 8 seeded
images (FP32 kernels); conv_i8_kernel launch i is then convolution i + 1
(model.0 runs in stem_i8_kernel): 0 model.1, 1 model.2.cv1, ...
"""
import argparse
import ctypes as C
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import yb_weights as yw  # noqa: E402
import yolo_b200 as yb  # noqa: E402

KINDS = ["conv_tc", "stem", "dwconv", "maxpool", "attention", "decode", "topk"]
KINDS_I8 = ["conv_i8", "stem_i8", "dw3x3_i8", "pool_cat", "attn_i8", "decode", "topk"]


class OpStat(C.Structure):
    _fields_ = [("kind", C.c_int), ("step", C.c_int), ("ms", C.c_double), ("flops", C.c_double),
                ("bytes", C.c_double)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--hw", type=int, default=640)
    ap.add_argument("--width", default="n", choices=["n", "s"])
    ap.add_argument("--ops", action="store_true")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--int8", action="store_true")
    a = ap.parse_args()
    with tempfile.TemporaryDirectory() as td:
        w = os.path.join(td, f"yolo26{a.width}.bin")
        yw.write_bin(w, yw.random_state(a.width, 0))
        m = yb.Model(w)
        if a.int8:
            m.calibrate_int8(yw.make_batch(range(10000, 10008), a.hw, a.hw))
        m.forward(yw.make_batch(range(1, a.batch + 1), a.hw, a.hw))
        if a.ops:
            L = yb.lib()
            n = C.c_int()
            yb.check(L.yb_cuda_profile_ops(m.ctx, a.batch, a.hw, a.hw, 300, 0, None, 0, C.byref(n)), "profile")
            st = (OpStat * n.value)()
            yb.check(L.yb_cuda_profile_ops(m.ctx, a.batch, a.hw, a.hw, 300, a.reps, st, n.value, C.byref(n)),
                     "profile")
            tot = sum(s.ms for s in st)
            for i, s in enumerate(st):
                print(f"{i:3d} {(KINDS_I8 if a.int8 else KINDS)[s.kind]:9s} step{s.step:2d} {s.ms:8.4f} ms {100 * s.ms / tot:5.1f}% "
                      f"{s.bytes / 1e6:9.1f} MB {s.bytes / s.ms / 1e6:8.1f} GB/s {s.flops / s.ms / 1e9:8.1f} TF/s")
            print(f"total {tot:.4f} ms for {a.batch} images")
        m.close()
    print("ok")


if __name__ == "__main__":
    main()
