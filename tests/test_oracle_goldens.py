"""Pins the CPU oracle to the reference's own golden vectors (tests/data/*.bin
of phucb2/yolo-baremetal, copied under tests/golden/), with the tolerance the
reference's tests/test_core.c uses (max abs < 5e-4, test_core.c:307,360,460)."""
import numpy as np
import pytest

from conftest import golden, max_abs


def _oracle_from(records, prefix, rename):
    from oracle import Oracle

    o = Oracle(nc=80)
    for k, v in records.items():
        name = rename(k)
        if name is None:
            continue
        o.add(f"{prefix}.{name}", v if v.ndim else v.reshape(1))
    return o


def _c3k2_name(tag):
    # <tag>_cv1_weight -> cv1.conv.weight, <tag>_m0_cv2_bias -> m.0.cv2.conv.bias
    def f(k):
        if not k.startswith(tag + "_") or k.endswith("_input") or k.endswith("_output"):
            return None
        parts = k[len(tag) + 1:].split("_")
        kind = parts[-1]
        mod = parts[:-1]
        if mod[0].startswith("m") and mod[0][1:].isdigit():
            mod = ["m", mod[0][1:]] + mod[1:]
        return ".".join(mod) + f".conv.{kind}"
    return f


@pytest.mark.parametrize("fname,tag,n,shortcut", [("c3k2_unit.bin", "unit", 2, 1), ("c3k2_yaml.bin", "yaml", 2, 0)])
def test_c3k2_golden(fname, tag, n, shortcut):
    """test_core.c:231-314: C3k2(64,64,n=2,shortcut) and C3k2(256,256,n=2,e=0.25)."""
    r = golden(fname)
    o = _oracle_from(r, "X", _c3k2_name(tag))
    x, want = r[f"{tag}_input"], r[f"{tag}_output"]
    out = np.zeros_like(want)
    st = o.lib().orc_c3k2(o.h, b"X", n, shortcut, x.reshape(-1), x.shape[1], x.shape[2], x.shape[3], out.reshape(-1),
                          want.shape[1])
    assert st == 0
    assert max_abs(out, want) < 5e-4


@pytest.mark.parametrize("fname,shortcut", [("sppf_test.bin", 0), ("sppf_shortcut.bin", 1)])
def test_sppf_golden(fname, shortcut):
    """test_core.c:316-366: SPPF k=5, 3 pools, without and with the residual."""
    r = golden(fname)
    rename = lambda k: None if k in ("sppf_input", "sppf_output") else k[5:].replace("_weight", ".conv.weight").replace("_bias", ".conv.bias")  # noqa: E731
    o = _oracle_from(r, "X", rename)
    x, want = r["sppf_input"], r["sppf_output"]
    out = np.zeros_like(want)
    st = o.lib().orc_sppf(o.h, b"X", 5, 3, shortcut, x.reshape(-1), x.shape[1], x.shape[2], x.shape[3],
                          out.reshape(-1), want.shape[1])
    assert st == 0
    assert max_abs(out, want) < 5e-4


def test_c2psa_golden():
    """test_core.c:368-465: C2PSA(128,128,n=2), 8x8 (64 tokens), 1 head."""
    r = golden("c2psa_test.bin")

    def rename(k):
        if k in ("c2psa_input", "c2psa_output"):
            return None
        s = k[len("c2psa_"):]
        kind = "weight" if s.endswith("_weight") else "bias"
        base = s[: -len(kind) - 1]
        if base in ("cv1", "cv2"):
            return f"{base}.conv.{kind}"
        blk, part = base.split("_")
        path = {"qkv": "attn.qkv", "proj": "attn.proj", "pe": "attn.pe", "ffn0": "ffn.0", "ffn1": "ffn.1"}[part]
        return f"m.{blk[1:]}.{path}.conv.{kind}"

    o = _oracle_from(r, "X", rename)
    x, want = r["c2psa_input"], r["c2psa_output"]
    out = np.zeros_like(want)
    st = o.lib().orc_c2psa(o.h, b"X", 2, x.reshape(-1), x.shape[1], x.shape[2], x.shape[3], out.reshape(-1),
                           want.shape[1])
    assert st == 0
    assert max_abs(out, want) < 5e-4


def test_conv_golden():
    """tests/data/conv_test.bin: 3x3 stride 2, 32->64 at 64x64, no bias."""
    r = golden("conv_test.bin")
    from oracle import Oracle

    o = Oracle(nc=80)
    o.add("X.conv.weight", r["weight"])
    x, want = r["input"], r["output"]
    out = np.zeros_like(want)
    st = o.lib().orc_conv_block(o.h, b"X", x.reshape(-1), 32, 64, 64, 2, 1, 0, out.reshape(-1))
    assert st == 0
    assert max_abs(out, want) < 1e-5


def test_c3k2_c3k_unfused_golden():
    """tests/data/c3k2_test.bin: an unfused C3k2(64,64,n=2,c3k=True) at 32x32
    with Conv+BN records; the oracle folds BN (utils.c:81-106) and runs the
    C3k chain."""
    r = golden("c3k2_test.bin")
    o = _oracle_from(r, "X", lambda k: None if k in ("input", "output") else k)
    o.fold()
    assert o.get("X.cv1.bn.weight") is None and o.get("X.cv1.conv.bias") is not None
    x, want = r["input"], r["output"]
    out = np.zeros_like(want)
    st = o.lib().orc_c3k2_c3k(o.h, b"X", x.reshape(-1), 64, 32, 32, out.reshape(-1), 64)
    assert st == 0
    assert max_abs(out, want) < 5e-4


def test_postprocess_known_answer():
    """test_core.c:491-510: N=1, nc=3 -> the best class is 1 with score 0.5."""
    from oracle import Oracle

    pred = np.array([0, 0, 10, 10, 0.2, 0.5, 0.3], dtype=np.float32)
    out = Oracle.postprocess(pred, nc=3, max_det=3, cap=3)
    assert abs(out[0, 0]) < 1e-5 and abs(out[0, 4] - 0.5) < 1e-5 and abs(out[0, 5] - 1.0) < 1e-5
