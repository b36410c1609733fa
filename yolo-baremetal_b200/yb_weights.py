"""Seeded random-init YOLO26 weights in the converter's .bin layout, and seeded inputs.

The .bin layout is the one tools/converter.py writes and src/utils.c:40-64 /
src/model.c:182-198 read (phucb2/yolo-baremetal): little-endian int32 nc,
int32 count, then per tensor int32 name_len, name bytes, int32 ndim,
int32 dims[ndim], float32 data.  Names are sorted (converter.py:116).

Tensor names and shapes follow the Ultralytics YOLO26 modules as the reference
wires them (model.c:208-665, detect.c:168-232): unfused Conv+BN records
(`<p>.conv.weight`, `<p>.bn.{weight,bias,running_mean,running_var,
num_batches_tracked}`), plain Conv2d heads (`<p>.weight`, `<p>.bias`), and
both the `cv2/cv3` and the `one2one_cv2/one2one_cv3` Detect branches (the
reference uses one2one when present, detect.c:297-299).

Init (the benchmark's stated recipe): conv weights Kaiming-normal
N(0, 2/fan_in); BN gamma = 1 + U(-0.1, 0.1), beta and running_mean ~ N(0, 0.1),
running_var ~ U(0.5, 1.5); plain Conv2d bias ~ N(0, 0.1).  `cls_scale`
multiplies the final class Conv2d weights and bias (a value like 0.01 keeps the
sigmoid scores away from saturation, so top-k order is decided by scores
rather than ties).
"""
from __future__ import annotations

import struct
from collections import OrderedDict

import numpy as np

# Ultralytics scale constants (depth, width, max_channels) from yolo26.yaml.
SCALES = {"n": (0.50, 0.25, 1024), "s": (0.50, 0.50, 1024)}


def _div8(x: float) -> int:
    return int(np.ceil(x / 8) * 8)


def yolo26_spec(scale: str = "n", nc: int = 80):
    """List of (prefix, kind, shape) for every parameterised module.

    kind: "conv" (Conv2d + BatchNorm), "plain" (Conv2d with bias).
    shape: (co, ci, kh, kw).
    """
    depth, width, max_ch = SCALES[scale]
    ch = lambda c: _div8(min(c, max_ch) * width)  # noqa: E731
    nrep = lambda r: max(round(r * depth), 1) if r > 1 else r  # noqa: E731
    spec = []

    def conv(p, ci, co, k=1):
        spec.append((p, "conv", (co, ci, k, k)))

    def dw(p, c, k=3):
        spec.append((p, "conv", (c, 1, k, k)))

    def bottleneck(p, c1, c2, e=0.5, k=3):
        c_ = int(c2 * e)
        conv(f"{p}.cv1", c1, c_, k)
        conv(f"{p}.cv2", c_, c2, k)

    def c3k(p, c1, c2, n=2, e=0.5):
        c_ = int(c2 * e)
        conv(f"{p}.cv1", c1, c_)
        conv(f"{p}.cv2", c1, c_)
        conv(f"{p}.cv3", 2 * c_, c2)
        for i in range(n):
            bottleneck(f"{p}.m.{i}", c_, c_, e=1.0)

    def psablock(p, c):
        heads = max(c // 64, 1)
        kd = int((c // heads) * 0.5)
        conv(f"{p}.attn.qkv", c, c + 2 * kd * heads)
        conv(f"{p}.attn.proj", c, c)
        dw(f"{p}.attn.pe", c)
        conv(f"{p}.ffn.0", c, 2 * c)
        conv(f"{p}.ffn.1", 2 * c, c)

    def c3k2(li, c1, c2, n, c3k_=False, e=0.5, attn=False):
        p = f"model.{li}"
        c = int(c2 * e)
        conv(f"{p}.cv1", c1, 2 * c)
        conv(f"{p}.cv2", (2 + n) * c, c2)
        for i in range(n):
            if attn:
                bottleneck(f"{p}.m.{i}.0", c, c)
                psablock(f"{p}.m.{i}.1", c)
            elif c3k_:
                c3k(f"{p}.m.{i}", c, c, 2)
            else:
                bottleneck(f"{p}.m.{i}", c, c)

    n2 = nrep(2)
    c0, c1_, c3_, c5, c7 = ch(64), ch(128), ch(256), ch(512), ch(1024)
    conv("model.0", 3, c0, 3)
    conv("model.1", c0, c1_, 3)
    c2o = ch(256)
    c3k2(2, c1_, c2o, n2, False, 0.25)
    conv("model.3", c2o, c3_, 3)
    c4o = ch(512)
    c3k2(4, c3_, c4o, n2, False, 0.25)
    conv("model.5", c4o, c5, 3)
    c3k2(6, c5, ch(512), n2, True)
    conv("model.7", ch(512), c7, 3)
    c3k2(8, c7, ch(1024), n2, True)
    c9 = ch(1024)
    conv("model.9.cv1", c9, c9 // 2)
    conv("model.9.cv2", (c9 // 2) * 4, c9)
    c10 = ch(1024)
    cc = int(c10 * 0.5)
    conv("model.10.cv1", c9, 2 * cc)
    conv("model.10.cv2", 2 * cc, c10)
    for i in range(n2):
        psablock(f"model.10.m.{i}", cc)
    c13 = ch(512)
    c3k2(13, c10 + ch(512), c13, n2, True)
    c16 = ch(256)
    c3k2(16, c13 + c4o, c16, n2, True)
    conv("model.17", c16, ch(256), 3)
    c19 = ch(512)
    c3k2(19, ch(256) + c13, c19, n2, True)
    conv("model.20", c19, ch(512), 3)
    c22 = ch(1024)
    c3k2(22, ch(512) + c10, c22, 1, True, 0.5, attn=True)
    feats = (c16, c19, c22)
    c2d = max(16, feats[0] // 4, 4)
    c3d = max(feats[0], min(nc, 100))
    for br in ("cv2", "one2one_cv2"):
        for i, x in enumerate(feats):
            p = f"model.23.{br}.{i}"
            conv(f"{p}.0", x, c2d, 3)
            conv(f"{p}.1", c2d, c2d, 3)
            spec.append((f"{p}.2", "plain", (4, c2d, 1, 1)))
    for br in ("cv3", "one2one_cv3"):
        for i, x in enumerate(feats):
            p = f"model.23.{br}.{i}"
            dw(f"{p}.0.0", x)
            conv(f"{p}.0.1", x, c3d)
            dw(f"{p}.1.0", c3d)
            conv(f"{p}.1.1", c3d, c3d)
            spec.append((f"{p}.2", "plain", (nc, c3d, 1, 1)))
    return spec


def random_state(scale: str = "n", seed: int = 0, nc: int = 80, cls_scale: float = 1.0) -> "OrderedDict[str, np.ndarray]":
    """Unfused state dict (Conv + BN records), seeded with numpy PCG64."""
    rng = np.random.default_rng(seed)
    sd: dict[str, np.ndarray] = {}
    for prefix, kind, (co, ci, kh, kw) in yolo26_spec(scale, nc):
        fan_in = ci * kh * kw
        w = rng.normal(0.0, np.sqrt(2.0 / fan_in), size=(co, ci, kh, kw)).astype(np.float32)
        if kind == "conv":
            sd[f"{prefix}.conv.weight"] = w
            sd[f"{prefix}.bn.weight"] = (1.0 + rng.uniform(-0.1, 0.1, co)).astype(np.float32)
            sd[f"{prefix}.bn.bias"] = rng.normal(0.0, 0.1, co).astype(np.float32)
            sd[f"{prefix}.bn.running_mean"] = rng.normal(0.0, 0.1, co).astype(np.float32)
            sd[f"{prefix}.bn.running_var"] = rng.uniform(0.5, 1.5, co).astype(np.float32)
            sd[f"{prefix}.bn.num_batches_tracked"] = np.zeros((), dtype=np.float32)
        else:
            b = rng.normal(0.0, 0.1, co).astype(np.float32)
            if "cv3." in prefix:  # final class Conv2d of a cv3 / one2one_cv3 branch
                w = (w * np.float32(cls_scale)).astype(np.float32)
                b = (b * np.float32(cls_scale)).astype(np.float32)
            sd[f"{prefix}.weight"] = w
            sd[f"{prefix}.bias"] = b
    return OrderedDict(sorted(sd.items(), key=lambda kv: kv[0]))


def write_bin(path: str, state: "OrderedDict[str, np.ndarray]", nc: int = 80) -> None:
    """Writes records in the converter's layout (converter.py:120-131)."""
    with open(path, "wb") as f:
        f.write(struct.pack("<ii", nc, len(state)))
        for name, arr in state.items():
            nb = name.encode("ascii")
            f.write(struct.pack("<i", len(nb)))
            f.write(nb)
            f.write(struct.pack("<i", arr.ndim))
            for d in arr.shape:
                f.write(struct.pack("<i", int(d)))
            f.write(np.ascontiguousarray(arr, dtype="<f4").tobytes())


def read_bin(path: str):
    """Parses a .bin file into (nc, OrderedDict name -> array)."""
    data = open(path, "rb").read()
    nc, count = struct.unpack_from("<ii", data, 0)
    off = 8
    out: "OrderedDict[str, np.ndarray]" = OrderedDict()
    for _ in range(count):
        (nl,) = struct.unpack_from("<i", data, off)
        off += 4
        name = data[off : off + nl].decode("ascii")
        off += nl
        (nd,) = struct.unpack_from("<i", data, off)
        off += 4
        dims = struct.unpack_from(f"<{nd}i", data, off)
        off += 4 * nd
        n = int(np.prod(dims)) if nd else 1
        arr = np.frombuffer(data, dtype="<f4", count=n, offset=off).reshape(dims if nd else ())
        off += 4 * n
        out[name] = arr.copy()
    return nc, out


def read_records(path: str):
    """Parses a file of bare records (stage dumps, golden fixtures)."""
    data = open(path, "rb").read()
    off = 0
    out: "OrderedDict[str, np.ndarray]" = OrderedDict()
    while off < len(data):
        (nl,) = struct.unpack_from("<i", data, off)
        off += 4
        name = data[off : off + nl].decode("ascii")
        off += nl
        (nd,) = struct.unpack_from("<i", data, off)
        off += 4
        dims = struct.unpack_from(f"<{nd}i", data, off)
        off += 4 * nd
        n = int(np.prod(dims)) if nd else 1
        out[name] = np.frombuffer(data, dtype="<f4", count=n, offset=off).reshape(dims if nd else ()).copy()
        off += 4 * n
    return out


def make_input(seed: int, h: int = 640, w: int = 640) -> np.ndarray:
    """One image [1, 3, h, w] float32 ~ U[0, 1) from numpy PCG64(seed)."""
    rng = np.random.default_rng(seed)
    return rng.random((1, 3, h, w), dtype=np.float32)


def make_batch(seeds, h: int = 640, w: int = 640) -> np.ndarray:
    return np.concatenate([make_input(s, h, w) for s in seeds], axis=0)
