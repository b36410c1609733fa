"""The reference's golden vectors (tests/data/*.bin of phucb2/yolo-baremetal,
copied under tests/golden/) run through this library's layers.h entry points
on the GPU, with the tolerance of the reference's tests/test_core.c (max abs
< 5e-4, test_core.c:307,360,460): C3k2 (two variants), SPPF (with and without
the residual), C2PSA with two PSA blocks, and the unfused C3k2/C3k chain
composed from conv_block_forward, c3_forward and concat_forward with BatchNorm
folded by the library's fold_bn.  Blocks without a golden (bottleneck,
psablock, C3) are compared with the CPU oracle."""
import numpy as np
import pytest

from conftest import golden, max_abs

pytestmark = pytest.mark.gpu

GOLDEN_TOL = 5e-4


def _tv(a):
    import yolo_b200 as yb

    return yb.tensor_view(np.ascontiguousarray(a, dtype=np.float32))


def _arr(tensors):
    import yolo_b200 as yb

    arr = (yb.Tensor * len(tensors))(*tensors)
    arr._views = list(tensors)  # the copies in the array point into these views' arrays
    return arr


def _ref(x):
    import yolo_b200 as yb

    return yb.C.byref(x)


def _buffers(n=8):
    """Scratch tensor array the reference's signatures take; the device path
    leaves it untouched."""
    return _arr([_tv(np.zeros(8, np.float32)) for _ in range(n)])


@pytest.mark.parametrize("fname,tag,shortcut", [("c3k2_unit.bin", "unit", True), ("c3k2_yaml.bin", "yaml", False)])
def test_c3k2_golden_gpu(fname, tag, shortcut):
    """test_core.c:231-314 through c3k2_forward."""
    import yolo_b200 as yb

    r = golden(fname)
    x, want = r[f"{tag}_input"], r[f"{tag}_output"]
    n = 2
    bw = []
    for i in range(n):
        for part in ("cv1_weight", "cv1_bias", "cv2_weight", "cv2_bias"):
            bw.append(_tv(r[f"{tag}_m{i}_{part}"]))
    out = np.zeros_like(want)
    bwa = _arr(bw)
    st = yb.lib().c3k2_forward(_ref(_tv(out)), _ref(_tv(x)), n, yb.C.c_bool(shortcut),
                               _ref(_tv(r[f"{tag}_cv1_weight"])), _ref(_tv(r[f"{tag}_cv1_bias"])),
                               _ref(_tv(r[f"{tag}_cv2_weight"])), _ref(_tv(r[f"{tag}_cv2_bias"])), bwa, _buffers())
    yb.check(st, "c3k2_forward")
    err = max_abs(out, want)
    print(f"{fname}: max abs err {err:.3e}")
    assert err < GOLDEN_TOL


@pytest.mark.parametrize("fname,shortcut", [("sppf_test.bin", False), ("sppf_shortcut.bin", True)])
def test_sppf_golden_gpu(fname, shortcut):
    """test_core.c:316-366 through sppf_forward (k=5, 3 pools)."""
    import yolo_b200 as yb

    r = golden(fname)
    x, want = r["sppf_input"], r["sppf_output"]
    out = np.zeros_like(want)
    st = yb.lib().sppf_forward(_ref(_tv(out)), _ref(_tv(x)), _ref(_tv(r["sppf_cv1_weight"])),
                               _ref(_tv(r["sppf_cv1_bias"])), _ref(_tv(r["sppf_cv2_weight"])),
                               _ref(_tv(r["sppf_cv2_bias"])), 5, 3, yb.C.c_bool(shortcut), _buffers())
    yb.check(st, "sppf_forward")
    err = max_abs(out, want)
    print(f"{fname}: max abs err {err:.3e}")
    assert err < GOLDEN_TOL


def test_c2psa_golden_gpu():
    """test_core.c:368-465 through c2psa_forward: C2PSA(128,128,n=2), 8x8, 1 head."""
    import yolo_b200 as yb

    r = golden("c2psa_test.bin")
    x, want = r["c2psa_input"], r["c2psa_output"]
    psa = []
    for i in range(2):
        for part in ("qkv", "proj", "pe", "ffn0", "ffn1"):
            psa.append(_tv(r[f"c2psa_m{i}_{part}_weight"]))
            psa.append(_tv(r[f"c2psa_m{i}_{part}_bias"]))
    out = np.zeros_like(want)
    st = yb.lib().c2psa_forward(_ref(_tv(out)), _ref(_tv(x)), 2, yb.C.c_float(0.5), yb.C.c_float(0.5),
                                _ref(_tv(r["c2psa_cv1_weight"])), _ref(_tv(r["c2psa_cv1_bias"])),
                                _ref(_tv(r["c2psa_cv2_weight"])), _ref(_tv(r["c2psa_cv2_bias"])), _arr(psa),
                                _buffers())
    yb.check(st, "c2psa_forward")
    err = max_abs(out, want)
    print(f"c2psa_test.bin: max abs err {err:.3e}")
    assert err < GOLDEN_TOL


def _fold(r, prefix):
    """Conv+BN records -> (weight, bias) folded by the library's fold_bn."""
    import yolo_b200 as yb

    w = np.array(r[f"{prefix}.conv.weight"], dtype=np.float32, copy=True)
    b = np.zeros(w.shape[0], dtype=np.float32)
    tw, tb = _tv(w), _tv(b)
    yb.lib().fold_bn(_ref(tw), _ref(tb), _ref(_tv(r[f"{prefix}.bn.weight"])), _ref(_tv(r[f"{prefix}.bn.bias"])),
                     _ref(_tv(r[f"{prefix}.bn.running_mean"])), _ref(_tv(r[f"{prefix}.bn.running_var"])))
    return w, b


def _conv_block(x, w, b, stride=1, act=True):
    import yolo_b200 as yb

    k = w.shape[2]
    pad = (k - 1) // 2
    H, W = x.shape[2], x.shape[3]
    out = np.zeros((1, w.shape[0], (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1), np.float32)
    yb.check(yb.lib().conv_block_forward(_ref(_tv(out)), _ref(_tv(x)), _ref(_tv(w)), _ref(_tv(b)),
                                         yb.ConvParams(stride, pad, 1), yb.C.c_bool(act)), "conv_block_forward")
    return out


def _concat(a, b):
    import yolo_b200 as yb

    out = np.zeros((1, a.shape[1] + b.shape[1], a.shape[2], a.shape[3]), np.float32)
    yb.check(yb.lib().concat_forward(_ref(_tv(out)), _ref(_tv(a)), _ref(_tv(b)), 1), "concat_forward")
    return out


def test_c3k2_c3k_unfused_golden_gpu():
    """tests/data/c3k2_test.bin: C3k2(64,64,n=2,c3k=True) at 32x32 from raw
    Conv+BN records: cv1 -> halves (a, b) -> two C3k blocks chained on b
    (c3_forward, 2 shortcut bottlenecks each) -> concat(a, b, m0, m1) -> cv2."""
    import yolo_b200 as yb

    r = golden("c3k2_test.bin")
    x, want = r["input"], r["output"]
    y = _conv_block(x, *_fold(r, "cv1"))
    c = y.shape[1] // 2
    parts = [y[:, :c].copy(), y[:, c:].copy()]
    cur = parts[1]
    for i in range(2):
        p = f"m.{i}"
        cv1, cv2, cv3 = _fold(r, f"{p}.cv1"), _fold(r, f"{p}.cv2"), _fold(r, f"{p}.cv3")
        bw = []
        for j in range(2):
            for t in _fold(r, f"{p}.m.{j}.cv1") + _fold(r, f"{p}.m.{j}.cv2"):
                bw.append(_tv(t))
        out = np.zeros((1, cv3[0].shape[0], cur.shape[2], cur.shape[3]), np.float32)
        st = yb.lib().c3_forward(_ref(_tv(out)), _ref(_tv(cur)), _ref(_tv(cv1[0])), _ref(_tv(cv1[1])),
                                 _ref(_tv(cv2[0])), _ref(_tv(cv2[1])), _ref(_tv(cv3[0])), _ref(_tv(cv3[1])),
                                 _arr(bw), 2, yb.C.c_bool(True), _buffers())
        yb.check(st, "c3_forward")
        parts.append(out)
        cur = out
    cat = parts[0]
    for t in parts[1:]:
        cat = _concat(cat, t)
    got = _conv_block(cat, *_fold(r, "cv2"))
    err = max_abs(got, want)
    print(f"c3k2_test.bin: max abs err {err:.3e}")
    assert err < GOLDEN_TOL


def test_bottleneck_psablock_vs_oracle():
    """bottleneck_forward and psablock_forward against the CPU oracle's C3k2 and
    C2PSA building blocks, on the golden weights with a seeded input."""
    import yolo_b200 as yb
    from oracle import Oracle

    r = golden("c3k2_unit.bin")
    rng = np.random.default_rng(5)
    x = rng.standard_normal((1, 32, 24, 20), dtype=np.float32)
    out = np.zeros_like(x)
    tmp = _tv(np.zeros((1, 16, 24, 20), np.float32))
    st = yb.lib().bottleneck_forward(_ref(_tv(out)), _ref(_tv(x)), _ref(_tv(r["unit_m0_cv1_weight"])),
                                     _ref(_tv(r["unit_m0_cv1_bias"])), _ref(_tv(r["unit_m0_cv2_weight"])),
                                     _ref(_tv(r["unit_m0_cv2_bias"])), yb.C.c_bool(True), _ref(tmp))
    yb.check(st, "bottleneck_forward")
    o = Oracle(nc=80)
    for i, name in enumerate(("cv1", "cv2")):
        o.add(f"B.{name}.conv.weight", r[f"unit_m0_{name}_weight"])
        o.add(f"B.{name}.conv.bias", r[f"unit_m0_{name}_bias"])
    h = np.zeros((1, 16, 24, 20), np.float32)
    assert o.lib().orc_conv_block(o.h, b"B.cv1", x.reshape(-1), 32, 24, 20, 1, 1, 1, h.reshape(-1)) == 0
    ref = np.zeros_like(x)
    assert o.lib().orc_conv_block(o.h, b"B.cv2", h.reshape(-1), 16, 24, 20, 1, 1, 1, ref.reshape(-1)) == 0
    ref += x
    err = max_abs(out, ref)
    print(f"bottleneck: max abs err {err:.3e}")
    assert err < GOLDEN_TOL

    # psablock_forward: one PSA block of the C2PSA golden, checked against the
    # oracle's C2PSA with the same block (cv1/cv2 identity-free path: compare
    # the block alone by running c2psa with n_blocks=1 on both sides).
    r2 = golden("c2psa_test.bin")
    xb = rng.standard_normal((1, 64, 8, 8), dtype=np.float32)
    outb = np.zeros_like(xb)
    args = []
    for part in ("qkv", "proj", "pe", "ffn0", "ffn1"):
        args += [_ref(_tv(r2[f"c2psa_m0_{part}_weight"])), _ref(_tv(r2[f"c2psa_m0_{part}_bias"]))]
    st = yb.lib().psablock_forward(_ref(_tv(outb)), _ref(_tv(xb)), yb.C.c_bool(True), *args, 1, yb.C.c_float(0.5))
    yb.check(st, "psablock_forward")
    o2 = Oracle(nc=80)
    for part, path in (("qkv", "attn.qkv"), ("proj", "attn.proj"), ("pe", "attn.pe"), ("ffn0", "ffn.0"),
                       ("ffn1", "ffn.1")):
        o2.add(f"P.{path}.conv.weight", r2[f"c2psa_m0_{part}_weight"])
        o2.add(f"P.{path}.conv.bias", r2[f"c2psa_m0_{part}_bias"])
    refb = np.zeros_like(xb)
    assert o2.lib().orc_psablock(o2.h, b"P", xb.reshape(-1), 64, 8, 8, 1, refb.reshape(-1)) == 0
    err = max_abs(outb, refb)
    print(f"psablock: max abs err {err:.3e}")
    assert err < GOLDEN_TOL


@pytest.mark.parametrize("n_bottles", [0, 1, 2])
def test_c3_vs_oracle(n_bottles):
    """c3_forward (layers.c:156-189) against the oracle's C3 on the golden's
    first C3k block (BN folded), seeded input, 0-2 bottlenecks."""
    import yolo_b200 as yb
    from oracle import Oracle

    r = golden("c3k2_test.bin")
    o = Oracle(nc=80)
    keep = ("m.0.cv", *(f"m.0.m.{j}." for j in range(n_bottles)))
    for k, v in r.items():
        if k.startswith(keep) and v.ndim:
            o.add(f"X.{k}", v)
    o.fold()
    rng = np.random.default_rng(3 + n_bottles)
    x = rng.standard_normal((1, 32, 20, 28), dtype=np.float32)
    ref = np.zeros((1, 32, 20, 28), np.float32)
    assert o.lib().orc_c3(o.h, b"X.m.0", 1, x.reshape(-1), 32, 20, 28, ref.reshape(-1), 32) == 0
    cv1, cv2, cv3 = _fold(r, "m.0.cv1"), _fold(r, "m.0.cv2"), _fold(r, "m.0.cv3")
    bw = [_tv(t) for j in range(max(n_bottles, 1)) for t in _fold(r, f"m.0.m.{j}.cv1") + _fold(r, f"m.0.m.{j}.cv2")]
    out = np.zeros_like(ref)
    st = yb.lib().c3_forward(_ref(_tv(out)), _ref(_tv(x)), _ref(_tv(cv1[0])), _ref(_tv(cv1[1])), _ref(_tv(cv2[0])),
                             _ref(_tv(cv2[1])), _ref(_tv(cv3[0])), _ref(_tv(cv3[1])), _arr(bw), n_bottles,
                             yb.C.c_bool(True), _buffers())
    yb.check(st, "c3_forward")
    err = max_abs(out, ref)
    print(f"c3 n={n_bottles}: max abs err {err:.3e}")
    assert err < GOLDEN_TOL
