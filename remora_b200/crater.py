"""Synthetic crater images and the crater-CNN parameter layout.

Images: 64x64 single-channel f32, Gaussian background noise (sigma 0.1);
label-1 images carry 1-3 circular rims of radius 4-16 px (rim +0.8, dark
interior -0.3), label-0 images are noise only; labels alternate so every
batch is 50/50.  Seeded with numpy's PCG64.  The reference's own generator
(examples/crater_train.py:90-113) makes 32x32 images with one fixed ring;
this one follows the larger benchmark's description instead.

Parameters: one flat f32 vector, He-normal weights (std sqrt(2/fan_in)),
biases 0.01, laid out as
w1[16,1,3,3] b1[16] w2[32,16,3,3] b2[32] w3[64,8192] b3[64] w4[64] b4[1].
"""

from __future__ import annotations

import numpy as np

DATA_SEED = 1729
PARAMETER_SEED = 2718
IMAGE = 64

LAYOUT = (
    ("w1", (16, 1, 3, 3)),
    ("b1", (16,)),
    ("w2", (32, 16, 3, 3)),
    ("b2", (32,)),
    ("w3", (64, 8192)),
    ("b3", (64,)),
    ("w4", (64,)),
    ("b4", (1,)),
)
FAN_IN = {"w1": 9, "w2": 144, "w3": 8192, "w4": 64}


def offsets() -> dict[str, tuple[int, int, tuple[int, ...]]]:
    out = {}
    o = 0
    for name, shape in LAYOUT:
        n = int(np.prod(shape))
        out[name] = (o, o + n, shape)
        o += n
    return out


NPARAMS = sum(int(np.prod(s)) for _, s in LAYOUT)


def views(flat: np.ndarray) -> dict[str, np.ndarray]:
    """Named shaped views into a flat parameter (or gradient) vector."""
    return {k: flat[a:b].reshape(s) for k, (a, b, s) in offsets().items()}


def init_params(seed: int = PARAMETER_SEED) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    flat = np.empty(NPARAMS, dtype=np.float32)
    v = views(flat)
    for name, shape in LAYOUT:
        if name.startswith("w"):
            v[name][...] = rng.normal(0.0, np.sqrt(2.0 / FAN_IN[name]), shape).astype(np.float32)
        else:
            v[name][...] = 0.01
    return flat


def make_batch(count: int, seed: int = DATA_SEED, start: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """`count` images [count, 1, 64, 64] and labels [count] (f32 0/1)."""
    rng = np.random.Generator(np.random.PCG64([seed, start]))
    imgs = rng.normal(0.0, 0.1, (count, 1, IMAGE, IMAGE)).astype(np.float32)
    labels = ((np.arange(start, start + count) % 2) == 0).astype(np.float32)
    yy, xx = np.mgrid[0:IMAGE, 0:IMAGE].astype(np.float32)
    for i in np.nonzero(labels)[0]:
        for _ in range(int(rng.integers(1, 4))):
            r = float(rng.uniform(4.0, 16.0))
            cy, cx = rng.uniform(r, IMAGE - 1 - r, 2)
            d = np.sqrt((yy - cy) ** 2 + (xx - cx) ** 2)
            img = imgs[i, 0]
            img[np.abs(d - r) <= 1.0] += 0.8
            img[d < r - 1.0] -= 0.3
    return imgs, labels
