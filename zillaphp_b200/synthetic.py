"""Seeded synthetic inputs and weights (the datasets are not available).

Counter-based Philox streams make the same seed give the same bytes on
every machine, so the library and the CPU oracle see identical inputs and
weights.  Weights are Kaiming-uniform U(+-sqrt(6/fan_in)) with zero bias;
the reference itself draws N(0, 1/in) through PHP's mt_rand
(src/NN/Layers/Linear.php:23-28, src/NN/Layers/Conv2D.php:25-44), which only
changes the starting point, not the step being compared.
"""
from __future__ import annotations

import numpy as np

from .configs import CONV, LINEAR, Workload


def rng(seed: int, stream: int = 0) -> np.random.Generator:
    return np.random.Generator(np.random.Philox(key=seed, counter=[0, 0, 0, stream]))


def init_params(w: Workload, seed: int = 1234) -> np.ndarray:
    """Flat parameters in Sequential::parameters() order: [W, b] per layer."""
    g = rng(seed, 1)
    parts = []
    for kind, a, b, _ in w.layers:
        if kind == CONV:
            bound = np.sqrt(6.0 / (a * 9))
            parts += [g.uniform(-bound, bound, size=b * a * 9), np.zeros(b)]
        elif kind == LINEAR:
            bound = np.sqrt(6.0 / a)
            parts += [g.uniform(-bound, bound, size=a * b), np.zeros(b)]
    return np.concatenate(parts).astype(np.float32)


def batch(w: Workload, n: int, seed: int = 1234, step: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """(x [n, C*H*W] float32, y [n] float-coded labels) for step `step`."""
    g = rng(seed, 1000 + step)
    if w.input_dist == "normal_m4_s2":
        x = g.normal(-4.0, 2.0, size=(n, w.in_features))
    else:
        x = g.random(size=(n, w.in_features))
    y = g.integers(0, w.classes, size=n)
    return x.astype(np.float32), y.astype(np.float32)
