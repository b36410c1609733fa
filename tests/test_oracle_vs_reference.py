"""Pins the CPU oracle to the reference itself: the reference's own C sources,
compiled from their files by oracle/Makefile into oracle/_ref/, run through its
public API (model_create / model_load_weights / model_forward_ex) on the same
seeded weights and inputs.  The oracle follows the reference's summation order,
so stage dumps, class logits and detections agree bit for bit."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.skipif(
    not os.path.exists(os.path.join(os.path.dirname(__file__), "..", "oracle", "_ref", "libyolo_ref.so")),
    reason="oracle/_ref not built (the reference sources were not available when build() ran)")


def _compare(weights, img, tmp_path, width_mult=1):
    import yb_weights as yw
    from oracle import Oracle, Reference

    o = Oracle(weights).forward(img, stages=True)
    stage_file = str(tmp_path / "ref_stages.bin")
    r = Reference.forward(weights, img, width_mult=width_mult, stage_path=stage_file)
    rs = yw.read_records(stage_file)
    assert list(rs.keys()) == list(o["stages"].keys())
    for k, v in o["stages"].items():
        assert np.array_equal(v, rs[k]), k
    assert np.array_equal(o["logits"], r["logits"])
    assert np.array_equal(o["dets"], r["dets"])


@pytest.mark.parametrize("hw,seed", [(64, 1), (128, 2), (96, 3)])
def test_n_width_bit_exact(weights_n0, tmp_path, hw, seed):
    import yb_weights as yw

    _compare(weights_n0, yw.make_input(seed, hw, hw), tmp_path)


def test_non_square_input(weights_n0, tmp_path):
    import yb_weights as yw

    _compare(weights_n0, yw.make_input(4, 64, 128), tmp_path)


def test_soft_weights(weights_n0_soft, tmp_path):
    import yb_weights as yw

    _compare(weights_n0_soft, yw.make_input(7, 128, 128), tmp_path)


def test_cv2_cv3_fallback(weights_n0_o2m, weights_n0_soft, tmp_path):
    """A checkpoint without the one-to-one Detect branches: the reference
    falls back to model.23.cv2 / cv3 (detect.c:297-299); so does the oracle,
    bit for bit, and the result differs from the one-to-one branches'."""
    import yb_weights as yw
    from oracle import Oracle

    img = yw.make_input(13, 128, 128)
    _compare(weights_n0_o2m, img, tmp_path)
    a = Oracle(weights_n0_o2m).forward(img)["dets"]
    b = Oracle(weights_n0_soft).forward(img)["dets"]
    assert not np.array_equal(a, b)


def test_s_width_bit_exact(weights_s0, tmp_path):
    """The s width (channels x2): the harness re-allocates the reference's
    model_t.buffers wider, since model_create sizes them for n."""
    import yb_weights as yw

    _compare(weights_s0, yw.make_input(5, 64, 64), tmp_path, width_mult=2)


def test_full_size_bit_exact(weights_n0, weights_s0, tmp_path):
    """The benchmark sizes: n width at 640x640 (400-token attention) and at
    1280x1280 (1600 tokens, 2 heads), and the s width at 1280x1280 (4 heads
    over 1600 tokens).  The three reference forwards run side by side in
    threads (the C calls release the GIL; the reference keeps no global
    state), each compared with the oracle stage by stage, on the logits and
    on the detections."""
    from concurrent.futures import ThreadPoolExecutor

    import yb_weights as yw
    from oracle import Oracle, Reference

    cases = [(weights_n0, 640, 1, 1), (weights_n0, 1280, 1, 9), (weights_s0, 1280, 2, 5)]

    def run_ref(i):
        w, hw, mult, seed = cases[i]
        path = str(tmp_path / f"ref_{i}.bin")
        r = Reference.forward(w, yw.make_input(seed, hw, hw), width_mult=mult, stage_path=path)
        return r, yw.read_records(path)

    with ThreadPoolExecutor(len(cases)) as ex:
        refs = list(ex.map(run_ref, range(len(cases))))
    for (w, hw, mult, seed), (r, rs) in zip(cases, refs):
        o = Oracle(w).forward(yw.make_input(seed, hw, hw), stages=True)
        assert list(rs.keys()) == list(o["stages"].keys())
        for k, v in o["stages"].items():
            assert np.array_equal(v, rs[k]), (hw, mult, k)
        assert np.array_equal(o["logits"], r["logits"]), (hw, mult)
        assert np.array_equal(o["dets"], r["dets"]), (hw, mult)


def test_postprocess_matches_reference():
    """Random predictions with many exact score ties: the oracle's explicit
    (score desc, index asc) order equals the reference's qsort output."""
    from oracle import Oracle, Reference

    rng = np.random.default_rng(0)
    N, nc = 2000, 80
    pred = rng.random((N, 4 + nc), dtype=np.float32)
    pred[:, 4:] = np.round(pred[:, 4:] * 8) / 8  # heavy ties
    for max_det, cap in [(300, 300), (300, 128), (5000, 1024)]:
        a = Oracle.postprocess(pred, nc, max_det, cap)
        b = Reference.postprocess(pred, nc, max_det, cap)
        assert np.array_equal(a, b), (max_det, cap)


def test_postprocess_edge_cases():
    from oracle import Oracle, Reference

    nc = 3
    for N in (0, 1, 2):
        pred = np.arange(N * (4 + nc), dtype=np.float32).reshape(N, 4 + nc) / 10
        a = Oracle.postprocess(pred, nc, 300, 4)
        b = Reference.postprocess(pred, nc, 300, 4) if N else np.zeros((4, 6), np.float32)
        assert np.array_equal(a, b)
