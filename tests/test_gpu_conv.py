"""Parity of the tcgen05 implicit-GEMM convolution (through conv_block_forward,
the reference's layers.h entry point) against the CPU oracle and the
reference's own conv golden vector."""
import numpy as np
import pytest

from conftest import golden, max_abs

pytestmark = pytest.mark.gpu

# The five YOLO26n backbone shapes of the conv sweep (ci, co, k, stride, H):
SWEEP = [(3, 16, 3, 2, 640), (16, 32, 3, 2, 320), (64, 64, 1, 1, 160), (128, 128, 3, 1, 40), (256, 256, 3, 1, 20)]
# Edge shapes: odd channel counts (padded to 4 on upload), N tails, two N tiles,
# K tails, tiny and non-square maps.
EDGE = [(2, 3, 1, 1, 2), (16, 4, 1, 1, 80), (80, 80, 1, 1, 40), (384, 128, 1, 1, 40), (256, 384, 1, 1, 24),
        (8, 16, 3, 1, 160), (48, 64, 1, 1, 36), (64, 64, 3, 2, 17), (32, 64, 3, 2, 64), (512, 256, 1, 1, 20)]


def _run(ci, co, k, stride, H, W=None, act=True, seed=0):
    import yolo_b200 as yb
    from oracle import Oracle

    W = W or H
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((1, ci, H, W), dtype=np.float32)
    w = (rng.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
    b = (rng.standard_normal(co) * 0.1).astype(np.float32)
    pad = (k - 1) // 2
    Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    out = np.zeros((1, co, Ho, Wo), dtype=np.float32)
    st = yb.lib().conv_block_forward(yb.C.byref(yb.tensor_view(out)), yb.C.byref(yb.tensor_view(x)),
                                     yb.C.byref(yb.tensor_view(w)), yb.C.byref(yb.tensor_view(b)),
                                     yb.ConvParams(stride, pad, 1), yb.C.c_bool(act))
    yb.check(st, "conv_block_forward")
    o = Oracle(nc=80)
    o.add("t.conv.weight", w)
    o.add("t.conv.bias", b)
    ref = np.zeros_like(out)
    assert o.lib().orc_conv_block(o.h, b"t", x.reshape(-1), ci, H, W, stride, pad, int(act), ref.reshape(-1)) == 0
    return out, ref


def _tol(ref, K):
    # split-bf16 products carry ~2^-16 relative error; allow growth with sqrt(K)
    return 3e-5 * max(1.0, float(np.abs(ref).max())) * max(1.0, np.sqrt(K / 64.0))


@pytest.mark.parametrize("ci,co,k,stride,H", SWEEP)
def test_conv_sweep_shapes(ci, co, k, stride, H):
    out, ref = _run(ci, co, k, stride, H)
    err = max_abs(out, ref)
    print(f"conv {ci}->{co} k{k} s{stride} @{H}: max abs err {err:.3e} (max |ref| {np.abs(ref).max():.2f})")
    assert err <= _tol(ref, ci * k * k)


# 3x3 stride-1 shapes of the resident-weight patch mode (16 x 8 output tiles):
# Ci = 16, 32, 48; Co 8-48; maps whose sides are not multiples of the tile.
PATCH = [(16, 8, 160, 160), (16, 16, 20, 20), (32, 32, 40, 40), (16, 32, 37, 29), (32, 16, 80, 72),
         (48, 48, 23, 41), (16, 16, 7, 5)]


@pytest.mark.parametrize("ci,co,H,W", PATCH)
def test_conv_patch_mode_shapes(ci, co, H, W):
    out, ref = _run(ci, co, 3, 1, H, W=W, act=True, seed=ci + co + H)
    err = max_abs(out, ref)
    print(f"conv {ci}->{co} 3x3 s1 @{H}x{W}: max abs err {err:.3e}")
    assert err <= _tol(ref, ci * 9)


@pytest.mark.parametrize("ci,co,k,stride,H", EDGE)
def test_conv_edge_shapes(ci, co, k, stride, H):
    out, ref = _run(ci, co, k, stride, H, act=(co % 2 == 0))
    err = max_abs(out, ref)
    print(f"conv {ci}->{co} k{k} s{stride} @{H}: max abs err {err:.3e}")
    assert err <= _tol(ref, ci * k * k)


@pytest.mark.parametrize("ci,co,k,stride,H", [(2, 3, 1, 1, 2), (16, 32, 3, 2, 64), (64, 64, 1, 1, 40)])
def test_conv_repeat_deterministic(ci, co, k, stride, H):
    """The device path has no atomics or races: repeated calls are bit-identical."""
    first, ref = _run(ci, co, k, stride, H)
    assert max_abs(first, ref) <= _tol(ref, ci * k * k)
    for _ in range(15):
        again, _ = _run(ci, co, k, stride, H)
        assert np.array_equal(again, first)


def test_conv_non_square():
    out, ref = _run(32, 48, 3, 1, 24, W=40)
    assert max_abs(out, ref) <= _tol(ref, 288)


def test_conv_golden_vector():
    """tests/data/conv_test.bin of the reference: 3x3 s2 32->64 @64x64, no bias."""
    import yolo_b200 as yb

    g = golden("conv_test.bin")
    x, w, want = g["input"], g["weight"], g["output"]
    out = np.zeros_like(want)
    st = yb.lib().conv2d_forward(yb.C.byref(yb.tensor_view(out)), yb.C.byref(yb.tensor_view(x)),
                                 yb.C.byref(yb.tensor_view(w)), None, yb.ConvParams(2, 1, 1))
    yb.check(st, "conv2d_forward")
    err = max_abs(out, want)
    print(f"conv_test.bin: max abs err {err:.3e}")
    assert err < 5e-4


def test_conv1x1_known_answer():
    """test_core.c:63-84: identity-like 1x1 conv with per-channel bias."""
    import yolo_b200 as yb

    x = np.arange(8, dtype=np.float32).reshape(1, 2, 2, 2)
    w = np.zeros((3, 2, 1, 1), dtype=np.float32)
    w[0, 0] = 1.0
    b = np.array([0.0, 1.0, 2.0], dtype=np.float32)
    out = np.zeros((1, 3, 2, 2), dtype=np.float32)
    yb.check(yb.lib().conv2d_forward(yb.C.byref(yb.tensor_view(out)), yb.C.byref(yb.tensor_view(x)),
                                     yb.C.byref(yb.tensor_view(w)), yb.C.byref(yb.tensor_view(b)),
                                     yb.ConvParams(1, 0, 1)), "conv2d_forward")
    want = np.concatenate([x[:, :1], np.ones((1, 1, 2, 2), np.float32), 2 * np.ones((1, 1, 2, 2), np.float32)], 1)
    assert max_abs(out, want) < 1e-5


def test_tensor_gemm_known_answer():
    """test_core.c:37-51: tensor_gemm vs a naive product, 5x7x4."""
    import yolo_b200 as yb

    M, N, K = 5, 7, 4
    A = ((np.arange(M * K) % 3) * 0.25 - 0.5).astype(np.float32)
    B = ((np.arange(K * N) % 5) * 0.1 - 0.2).astype(np.float32)
    Cm = np.zeros(M * N, dtype=np.float32)
    yb.check(yb.lib().tensor_gemm(Cm.ctypes.data_as(yb.C.POINTER(yb.C.c_float)),
                                  A.ctypes.data_as(yb.C.POINTER(yb.C.c_float)),
                                  B.ctypes.data_as(yb.C.POINTER(yb.C.c_float)), M, N, K, yb.C.c_float(1.0),
                                  yb.C.c_float(0.0)), "tensor_gemm")
    want = A.reshape(M, K).astype(np.float64) @ B.reshape(K, N).astype(np.float64)
    assert max_abs(Cm.reshape(M, N), want) < 1e-5
