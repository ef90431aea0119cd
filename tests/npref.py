"""Float64 numpy statement of one training step (test helper).

An independent check of the oracle's step driver: the same Sequential
(Conv2D 3x3 stride 1, ReLU, MaxPool 2x2/2 with first-maximum argmax, Linear
W[in, out]), softmax cross-entropy with the softmax_ce_dev gradient
(p - onehot)/B (native/cpu/training_ops.c:162-206) and SGD / Adam
(src/Optim/Adam.php:36-62).  Small sizes only.
"""
from __future__ import annotations

import numpy as np

CONV, RELU, POOL, LINEAR = 1, 2, 3, 4


def _conv(x, w, b, pad):
    B, C, H, W = x.shape
    oC = w.shape[0]
    xp = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    oH, oW = H + 2 * pad - 2, W + 2 * pad - 2
    cols = np.empty((B, C, 3, 3, oH, oW))
    for kh in range(3):
        for kw in range(3):
            cols[:, :, kh, kw] = xp[:, :, kh:kh + oH, kw:kw + oW]
    y = np.einsum("bckluv,ockl->bouv", cols, w) + b[None, :, None, None]
    return y, cols


def _conv_bwd(cols, w, g, pad, H, W):
    dw = np.einsum("bckluv,bouv->ockl", cols, g)
    db = g.sum(axis=(0, 2, 3))
    dcols = np.einsum("ockl,bouv->bckluv", w, g)
    B, C = cols.shape[:2]
    oH, oW = g.shape[2:]
    dxp = np.zeros((B, C, H + 2 * pad, W + 2 * pad))
    for kh in range(3):
        for kw in range(3):
            dxp[:, :, kh:kh + oH, kw:kw + oW] += dcols[:, :, kh, kw]
    return dxp[:, :, pad:pad + H, pad:pad + W], dw, db


def _pool(x):
    B, C, H, W = x.shape
    oH, oW = (H - 2) // 2 + 1, (W - 2) // 2 + 1
    win = np.stack([x[:, :, dh:dh + 2 * oH:2, dw:dw + 2 * oW:2] for dh in (0, 1) for dw in (0, 1)], axis=-1)
    # first maximum in (kh, kw) order: argmax returns the first occurrence
    k = np.argmax(win, axis=-1)
    return np.take_along_axis(win, k[..., None], -1)[..., 0], k


def _pool_bwd(g, k, shape):
    B, C, H, W = shape
    oH, oW = g.shape[2:]
    dx = np.zeros(shape)
    for j, (dh, dw) in enumerate(((0, 0), (0, 1), (1, 0), (1, 1))):
        dx[:, :, dh:dh + 2 * oH:2, dw:dw + 2 * oW:2] += np.where(k == j, g, 0.0)
    return dx


def step(layers, in_shape, params, x, y, opt, lr, t=1, m=None, v=None, betas=(0.9, 0.999, 1e-8)):
    """Returns (loss_sum, grads, new_params, m, v, pool_codes) in float64."""
    p = params.astype(np.float64)
    B = x.shape[0]
    a = x.astype(np.float64).reshape((B,) + tuple(in_shape))
    cache, off, codes = [], 0, []
    for kind, i, o, pad in layers:
        if kind == CONV:
            w = p[off:off + o * i * 9].reshape(o, i, 3, 3); b = p[off + o * i * 9: off + o * i * 9 + o]
            y_, cols = _conv(a, w, b, pad)
            cache.append((kind, a.shape, cols, w, off, pad)); off += o * i * 9 + o; a = y_
        elif kind == RELU:
            cache.append((kind, a > 0)); a = np.maximum(a, 0)
        elif kind == POOL:
            out, k = _pool(a); cache.append((kind, a.shape, k)); codes.append(k); a = out
        else:
            a2 = a.reshape(B, -1)
            w = p[off:off + i * o].reshape(i, o); b = p[off + i * o: off + i * o + o]
            cache.append((kind, a.shape, a2, w, off)); off += i * o + o; a = a2 @ w + b
    z = a
    zmax = z.max(axis=1, keepdims=True)
    e = np.exp(z - zmax)
    pr = e / e.sum(axis=1, keepdims=True)
    yi = y.astype(np.int64)
    loss = -np.log(pr[np.arange(B), yi]).sum()
    g = pr.copy(); g[np.arange(B), yi] -= 1.0; g /= B
    grads = np.zeros_like(p)
    for item in reversed(cache):
        kind = item[0]
        if kind == CONV:
            _, shp, cols, w, o0, pad = item
            gx, dw, db = _conv_bwd(cols, w, g, pad, shp[2], shp[3])
            grads[o0:o0 + dw.size] = dw.ravel(); grads[o0 + dw.size:o0 + dw.size + db.size] = db; g = gx
        elif kind == RELU:
            g = g * item[1]
        elif kind == POOL:
            g = _pool_bwd(g, item[2], item[1])
        else:
            _, shp, a2, w, o0 = item
            grads[o0:o0 + w.size] = (a2.T @ g).ravel(); grads[o0 + w.size:o0 + w.size + w.shape[1]] = g.sum(0)
            g = (g @ w.T).reshape(shp)
    if opt == 1:
        newp = p - lr * grads
    elif opt == 2:
        b1, b2, eps = betas
        m = np.zeros_like(p) if m is None else m
        v = np.zeros_like(p) if v is None else v
        m = b1 * m + (1 - b1) * grads
        v = b2 * v + (1 - b2) * grads ** 2
        newp = p - lr * (m / (1 - b1 ** t)) / (np.sqrt(v / (1 - b2 ** t)) + eps)
    else:
        newp = p
    return loss, grads, newp, m, v, codes


def normwise(a, b) -> float:
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))
