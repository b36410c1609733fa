"""The reference's own C callers, compiled unchanged against this repository's
headers and linked to libyolo_b200.so (oracle/Makefile, target `callers`):
the drop-in claim of the boundary, checked with the reference's code instead
of ctypes.

  * tests/test_core.c (phucb2/yolo-baremetal, main at test_core.c:512-534):
    every case, including the golden-vector fixtures at its own 5e-4
    tolerance, runs on the GPU through tensor_gemm / conv2d_forward /
    c3k2_forward / sppf_forward / c2psa_forward / detect_postprocess_from_pred
    and must report "all checks passed";
  * tests/dump_model_stages.c (main at dump_model_stages.c:98-178): its
    model_create / model_load_weights / model_forward_ex stage dump, written
    by this library's GPU forward, is compared with the CPU oracle's dump of
    the same seeded weights and input.

The binaries are built where the reference sources are mounted and travel
with the repository; without them the tests skip."""
import os
import shutil
import struct
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, ROOT
from parity import STAGE_RTOL, compare_dets, dets_ok, rel_err

pytestmark = pytest.mark.gpu

REF_BIN = os.path.join(ROOT, "oracle", "_ref")
FIXTURES = ["c3k2_unit.bin", "c3k2_yaml.bin", "sppf_test.bin", "sppf_shortcut.bin", "c2psa_test.bin"]


def _exe(name):
    path = os.path.join(REF_BIN, name)
    if not os.path.exists(path):
        pytest.skip(f"oracle/_ref/{name} not built (the reference sources were absent when build() ran)")
    return path


def test_reference_test_core(tmp_path):
    """test_core.c opens its fixtures as tests/data/<name> relative to the
    working directory (test_core.c:189-196): the golden copies are laid out
    that way in a scratch directory."""
    exe = _exe("test_core_b200")
    data = tmp_path / "tests" / "data"
    data.mkdir(parents=True)
    for n in FIXTURES:
        shutil.copyfile(os.path.join(GOLDEN, n), data / n)
    r = subprocess.run([exe], cwd=tmp_path, capture_output=True, text=True, timeout=600)
    print(r.stdout)
    print(r.stderr)
    assert r.returncode == 0, r.stderr
    assert "all checks passed" in r.stdout
    assert "SKIP" not in r.stderr, "a fixture case did not run"


def _write_record(path, name, arr):
    with open(path, "wb") as f:
        nb = name.encode()
        f.write(struct.pack("<i", len(nb)))
        f.write(nb)
        f.write(struct.pack("<i", arr.ndim))
        f.write(struct.pack(f"<{arr.ndim}i", *arr.shape))
        f.write(np.ascontiguousarray(arr, dtype="<f4").tobytes())


def test_reference_dump_model_stages(tmp_path, weights_n0):
    """dump_model_stages <input.bin> <out.bin> <weights.bin>: a 640x640
    single-tensor input (dump_model_stages.c:30-43), all 26 stage records
    from this library's forward against the oracle's."""
    import yb_weights as yw
    from oracle import Oracle

    exe = _exe("dump_model_stages_b200")
    img = yw.make_input(1, 640, 640)
    inp = tmp_path / "input.bin"
    out = tmp_path / "stages.bin"
    _write_record(inp, "stage_00_input", img)
    r = subprocess.run([exe, str(inp), str(out), weights_n0], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    print(r.stderr)
    assert r.returncode == 0, r.stderr
    got = yw.read_records(str(out))
    ref = Oracle(weights_n0).forward(img, stages=True)["stages"]
    assert list(got.keys()) == list(ref.keys())
    for name, want in ref.items():
        have = got[name]
        assert have.shape == want.shape, name
        if name.startswith("stage_24") or name.startswith("stage_25"):
            c = compare_dets(have.reshape(-1, 6), want.reshape(-1, 6))
            print(f"{name}: {c}")
            assert dets_ok(c), name
        else:
            e = rel_err(have, want)
            print(f"{name}: rel err {e:.2e}")
            assert e <= STAGE_RTOL, name
