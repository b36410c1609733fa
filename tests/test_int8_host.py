"""CPU checks of the INT8 scheme: the library's host quantiser equals the
oracle's independent restatement bit for bit, the round-half-even shift and
the fixed-point multipliers follow their definitions, and the oracle's INT8
convolution equals a plain-Python integer convolution on small cases."""
import numpy as np
import pytest

from int8_util import conv_oracle, make_layer, orc_lib, quantize_lib, quantize_oracle


@pytest.mark.parametrize("ci,co,k,act,bias", [(3, 16, 3, True, True), (16, 32, 3, True, True), (64, 64, 1, False, True),
                                              (40, 48, 3, True, False), (256, 256, 3, True, True)])
def test_quantiser_matches_oracle(ci, co, k, act, bias):
    lyr = make_layer(ci, co, k, 12, 10, seed=ci + co, act=act, bias=bias)
    a, b = quantize_lib(lyr), quantize_oracle(lyr)
    for key in ("wq", "bq", "mult", "shift"):
        assert np.array_equal(a[key], b[key]), key
    if act:
        assert np.array_equal(a["lut"], b["lut"])
    # The multiplier represents s_in * s_w / s_t to 31 bits.
    sw = np.abs(lyr["w"]).reshape(co, -1).max(1) / np.float32(127.0)
    ratio = float(lyr["s_in"]) * sw.astype(np.float64) / float(lyr["s_pre"] if act else lyr["s_out"])
    approx = a["mult"].astype(np.float64) * 2.0 ** (-a["shift"].astype(np.float64))
    assert np.all(np.abs(approx - ratio) <= ratio * 2.0 ** -30)
    assert np.all((a["mult"] >= 2**30) & (a["shift"] >= 1) & (a["shift"] <= 62))


def test_rshift_round_half_even():
    L = orc_lib()
    rng = np.random.default_rng(3)
    vals = [(5, 1), (7, 1), (-5, 1), (-7, 1), (6, 2), (10, 2), (-6, 2), (-10, 2), (0, 5), (-1, 1), (1, 1)]
    vals += [(int(v), int(s)) for v, s in zip(rng.integers(-2**60, 2**60, 200), rng.integers(1, 40, 200))]
    for v, s in vals:
        q, r = divmod(v, 1 << s)  # floor division
        half = 1 << (s - 1)
        want = q + 1 if (r > half or (r == half and q % 2 == 1)) else q
        assert L.orc_i8_rshift_rne(v, s) == want, (v, s)


def _conv_py(xq, q, k, stride, pad):
    B, H, W, ci = xq.shape
    co = q["wq"].shape[0]
    Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    xp = np.zeros((B, H + 2 * pad, W + 2 * pad, ci), np.int64)
    xp[:, pad:pad + H, pad:pad + W] = xq
    y = np.zeros((B, Ho, Wo, co), np.int8)
    w = q["wq"].astype(np.int64)
    for oy in range(Ho):
        for ox in range(Wo):
            patch = xp[:, oy * stride:oy * stride + k, ox * stride:ox * stride + k, :]  # B,k,k,ci
            acc = np.einsum("bijc,ocij->bo", patch, w) + q["bq"].astype(np.int64)
            for o in range(co):
                for bb in range(B):
                    p = int(acc[bb, o]) * int(q["mult"][o])
                    s = int(q["shift"][o])
                    fl, rem = divmod(p, 1 << s)
                    half = 1 << (s - 1)
                    v = fl + 1 if (rem > half or (rem == half and fl % 2 == 1)) else fl
                    if q["lut"] is not None:
                        y[bb, oy, ox, o] = q["lut"][min(max(v, -128), 127) + 128]
                    else:
                        y[bb, oy, ox, o] = min(max(v, -127), 127)
    return y


@pytest.mark.parametrize("ci,co,k,stride,act", [(5, 16, 3, 1, True), (8, 16, 3, 2, False), (20, 32, 1, 1, True)])
def test_oracle_conv_matches_python(ci, co, k, stride, act):
    lyr = make_layer(ci, co, k, 7, 6, B=2, seed=7 + ci, act=act)
    q = quantize_oracle(lyr)
    assert np.array_equal(conv_oracle(lyr["xq"], q, k, stride, lyr["pad"]), _conv_py(lyr["xq"], q, k, stride, lyr["pad"]))
