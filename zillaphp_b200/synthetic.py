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

from .configs import CONV, LINEAR, LmWorkload, Workload


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


def lm_layout(w: LmWorkload) -> list[tuple[str, tuple]]:
    """(name, shape) of the language model's flat parameters in
    TransformerLM::parameters() order (src/Transformers/TransformerLM.php:158-170)."""
    V, D, F = w.vocab, w.dim, w.ffn
    out = [("tok", (V, D)), ("pos", (w.max_seq, D)), ("lnf.g", (D,)), ("lnf.b", (D,)),
           ("head.W", (D, V)), ("head.b", (V,))]
    for l in range(w.layers):
        for p in ("q", "k", "v", "o"):
            out += [(f"b{l}.{p}.W", (D, D)), (f"b{l}.{p}.b", (D,))]
        out += [(f"b{l}.fc1.W", (D, F)), (f"b{l}.fc1.b", (F,)), (f"b{l}.fc2.W", (F, D)), (f"b{l}.fc2.b", (D,))]
        out += [(f"b{l}.ln1.g", (D,)), (f"b{l}.ln1.b", (D,)), (f"b{l}.ln2.g", (D,)), (f"b{l}.ln2.b", (D,))]
    return out


def lm_init_params(w: LmWorkload, seed: int = 1234, perturb: float = 0.0) -> np.ndarray:
    """The reference's initial distributions drawn from a Philox stream:
    embedding tables N(0, 0.01^2) (src/NN/Layers/Embedding.php:22-33), Linear
    weights N(0, 1/in) with zero bias (src/NN/Layers/Linear.php:20-30),
    LayerNorm gamma 1, beta 0 (src/NN/Layers/LayerNorm.php:23-27).
    `perturb` > 0 adds N(0, perturb^2) to every bias, gamma and beta, so a
    check exercises those paths with non-trivial values."""
    g = rng(seed, 2)
    parts = []
    for name, shape in lm_layout(w):
        n = int(np.prod(shape))
        if name in ("tok", "pos"):
            a = g.normal(0.0, 0.01, n)
        elif name.endswith(".W"):
            a = g.normal(0.0, np.sqrt(1.0 / shape[0]), n)
        elif name.endswith(".g"):
            a = np.ones(n)
        else:
            a = np.zeros(n)
        if perturb > 0 and not name.endswith(".W") and name not in ("tok", "pos"):
            a = a + g.normal(0.0, perturb, n)
        parts.append(a)
    return np.concatenate(parts).astype(np.float32)


def lm_batch(w: LmWorkload, batch: int, seq: int, seed: int = 1234, step: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """(tokens [batch*seq], targets [batch*seq]) as floats: uniform ids in
    [0, vocab), targets the inputs shifted by one."""
    g = rng(seed, 3000 + step)
    ids = g.integers(0, w.vocab, size=(batch, seq + 1))
    return ids[:, :-1].reshape(-1).astype(np.float32), ids[:, 1:].reshape(-1).astype(np.float32)
