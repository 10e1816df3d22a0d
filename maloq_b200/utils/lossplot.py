"""Loss curves as a PNG without a plotting library.

The reference saves a matplotlib figure of the training and validation losses next to its
checkpoints (``splittrainer.py:650-673``).  matplotlib is not a dependency here, so the curves
are rasterised with numpy (log10 of the loss against the epoch, one colour per series, light
grid lines at the decades) and encoded as an RGB PNG with zlib.
"""

from __future__ import annotations

import struct
import zlib

import numpy as np

COLOURS = {"train_node": (31, 119, 180), "train_edge": (255, 127, 14), "val_node": (44, 160, 44),
           "val_edge": (214, 39, 40)}


def encode_png(img):
    """[H, W, 3] uint8 -> PNG bytes (8-bit RGB, no filtering)."""
    img = np.ascontiguousarray(img, dtype=np.uint8)
    h, w, _ = img.shape
    raw = b"".join(b"\x00" + img[r].tobytes() for r in range(h))

    def chunk(tag, data):
        return struct.pack(">I", len(data)) + tag + data + struct.pack(">I", zlib.crc32(tag + data) & 0xFFFFFFFF)

    return (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, 8, 2, 0, 0, 0))
            + chunk(b"IDAT", zlib.compress(raw, 6)) + chunk(b"IEND", b""))


def _line(img, x0, y0, x1, y1, colour):
    n = int(max(abs(x1 - x0), abs(y1 - y0))) + 1
    xs = np.rint(np.linspace(x0, x1, n)).astype(int)
    ys = np.rint(np.linspace(y0, y1, n)).astype(int)
    h, w, _ = img.shape
    for dx in (0, 1):  # two pixels wide
        ok = (xs + dx >= 0) & (xs + dx < w) & (ys >= 0) & (ys < h)
        img[ys[ok], xs[ok] + dx] = colour


def render(history, width=640, height=400, margin=30):
    """RGB image of the loss series in ``history`` (keys of :data:`COLOURS`, lists per epoch)."""
    img = np.full((height, width, 3), 255, dtype=np.uint8)
    series = {k: np.asarray(v, dtype=np.float64) for k, v in history.items() if k in COLOURS and len(v)}
    vals = np.concatenate([v[np.isfinite(v) & (v > 0)] for v in series.values()]) if series else np.zeros(0)
    if vals.size == 0:
        return img
    lo, hi = np.floor(np.log10(vals.min())), np.ceil(np.log10(vals.max()))
    hi = max(hi, lo + 1)
    n_ep = max(len(v) for v in series.values())
    x = lambda i: margin + (width - 2 * margin) * (i / max(1, n_ep - 1))
    y = lambda v: height - margin - (height - 2 * margin) * (np.log10(v) - lo) / (hi - lo)
    for d in np.arange(lo, hi + 1):  # decade grid lines
        img[int(round(y(10.0 ** d))) - (1 if d == hi else 0), margin:width - margin] = (220, 220, 220)
    img[margin:height - margin, margin] = 0
    img[height - margin, margin:width - margin] = 0
    for k, v in series.items():
        pts = [(x(i), y(val)) for i, val in enumerate(v) if np.isfinite(val) and val > 0]
        for (x0, y0), (x1, y1) in zip(pts, pts[1:]):
            _line(img, x0, y0, x1, y1, COLOURS[k])
        for px, py in pts:
            r, c = int(round(py)), int(round(px))
            img[max(0, r - 2):r + 3, max(0, c - 2):c + 3] = COLOURS[k]
    return img


def save_loss_png(path, history):
    with open(path, "wb") as f:
        f.write(encode_png(render(history)))
    return path
