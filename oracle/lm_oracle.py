"""Float64 numpy restatement of ZillaPHP's Transformer LM training step
(TEST INFRASTRUCTURE ONLY: the checker for the library's language-model step).

Follows the reference:
  TransformerLM::forwardBatch         src/Transformers/TransformerLM.php:77-116
  TransformerBlock::forward (pre-LN)  src/Transformers/TransformerBlock.php:28-33
  MultiHeadAttention::forward         src/Attention/MultiHeadAttention.php:41-80
      per head: (Q K^T) * (1/sqrt(head_dim)), maskedFill(-1e9) on future keys,
      row softmax, times V; concat heads; output Linear
  FeedForward                         src/NN/Layers/FeedForward.php (fc1, ReLU, fc2)
  Tensor::layerNorm (+ backward)      src/Tensor/Tensor.php:636-735 (biased variance, eps 1e-5)
  Embedding::forward                  src/NN/Layers/Embedding.php:35-56 (one-hot @ table = row gather)
  softmax backward                    src/Tensor/Tensor.php:1184-1221
  maskedFill backward                 src/Tensor/Tensor.php:565-594 (zero on masked entries)
  loss                                softmax_ce_dev, native/cpu/training_ops.c:162-206
                                      (sum of -log p over rows; dlogits = (p - onehot) / rows)
  Adam                                src/Optim/Adam.php:36-62
  TransformerLM::forwardWithCache     src/Transformers/TransformerLM.php:124-151 (generation;
                                      forward_cached below: K/V cache, no causal mask)
The batched block-diagonal mask of forwardBatch (src/Tensor/Tensor.php:619-634)
is evaluated per sequence: masked scores are -1e9, whose softmax weight is
exactly 0, so attention never crosses sequences.

Parameters: one flat vector in TransformerLM::parameters() order
(src/Transformers/TransformerLM.php:158-170): token table, position table,
final LayerNorm (gamma, beta), head (W, b), then per block: attention
(Wq, bq, Wk, bk, Wv, bv, Wo, bo), FFN (W1, b1, W2, b2), ln1 (g, b), ln2 (g, b).
Linear weights are [in, out] (src/NN/Layers/Linear.php:14).
"""
from __future__ import annotations

import numpy as np


def layout(V, D, L, T, F):
    names = [("tok", (V, D)), ("pos", (T, D)), ("lnf.g", (D,)), ("lnf.b", (D,)),
             ("head.W", (D, V)), ("head.b", (V,))]
    for l in range(L):
        for p in ("q", "k", "v", "o"):
            names += [(f"b{l}.{p}.W", (D, D)), (f"b{l}.{p}.b", (D,))]
        names += [(f"b{l}.fc1.W", (D, F)), (f"b{l}.fc1.b", (F,)), (f"b{l}.fc2.W", (F, D)), (f"b{l}.fc2.b", (D,))]
        names += [(f"b{l}.ln1.g", (D,)), (f"b{l}.ln1.b", (D,)), (f"b{l}.ln2.g", (D,)), (f"b{l}.ln2.b", (D,))]
    return names


def unflatten(flat, V, D, L, T, F):
    out, off = {}, 0
    for name, shape in layout(V, D, L, T, F):
        n = int(np.prod(shape))
        out[name] = flat[off:off + n].reshape(shape)
        off += n
    return out


def flatten(d, V, D, L, T, F):
    return np.concatenate([d[name].ravel() for name, _ in layout(V, D, L, T, F)])


def _ln(x, g, b, eps=1e-5):
    mean = x.mean(1, keepdims=True)
    var = ((x - mean) ** 2).mean(1, keepdims=True)
    inv = 1.0 / np.sqrt(var + eps)
    xhat = (x - mean) * inv
    return xhat * g + b, (xhat, inv)


def _ln_bwd(gout, g, cache):
    xhat, inv = cache
    D = xhat.shape[1]
    gx = gout * g
    s1 = gx.sum(1, keepdims=True)
    s2 = (gx * xhat).sum(1, keepdims=True)
    dx = inv / D * (D * gx - s1 - xhat * s2)
    return dx, (gout * xhat).sum(0), gout.sum(0)


def attention(q, k, v, B, T, H):
    """q, k, v: [B*T, D] -> (out [B*T, D], probs [B, H, T, T])."""
    D = q.shape[1]
    dh = D // H
    scale = 1.0 / np.sqrt(dh)
    qh = q.reshape(B, T, H, dh).transpose(0, 2, 1, 3)
    kh = k.reshape(B, T, H, dh).transpose(0, 2, 1, 3)
    vh = v.reshape(B, T, H, dh).transpose(0, 2, 1, 3)
    s = np.einsum("bhid,bhjd->bhij", qh, kh) * scale
    future = np.triu(np.ones((T, T), bool), 1)
    s = np.where(future, -1e9, s)
    s = s - s.max(-1, keepdims=True)
    e = np.exp(s)
    p = e / e.sum(-1, keepdims=True)
    o = np.einsum("bhij,bhjd->bhid", p, vh)
    return o.transpose(0, 2, 1, 3).reshape(B * T, D), p


def attention_bwd(do, q, k, v, p, B, T, H):
    D = q.shape[1]
    dh = D // H
    scale = 1.0 / np.sqrt(dh)
    sh = lambda a: a.reshape(B, T, H, dh).transpose(0, 2, 1, 3)
    qh, kh, vh, doh = sh(q), sh(k), sh(v), sh(do)
    dv = np.einsum("bhij,bhid->bhjd", p, doh)
    dp = np.einsum("bhid,bhjd->bhij", doh, vh)
    ds = p * (dp - (dp * p).sum(-1, keepdims=True))       # softmax backward; masked entries: p = 0
    ds = ds * scale
    dq = np.einsum("bhij,bhjd->bhid", ds, kh)
    dk = np.einsum("bhij,bhid->bhjd", ds, qh)
    un = lambda a: a.transpose(0, 2, 1, 3).reshape(B * T, D)
    return un(dq), un(dk), un(dv)


def step(flat, tokens, targets, V, D, H, L, T, F, opt="adam", lr=3e-4, t=1, m=None, v=None,
         betas=(0.9, 0.999, 1e-8)):
    """One training step.  tokens, targets: [B, T] ints.
    Returns (loss_sum, grads_flat, new_flat, m, v, logits)."""
    B, Ts = tokens.shape
    N = B * Ts
    P = unflatten(np.asarray(flat, np.float64), V, D, L, T, F)
    ids = tokens.reshape(N).astype(np.int64)
    pos = np.tile(np.arange(Ts), B)
    x = P["tok"][ids] + P["pos"][pos]
    caches = []
    for l in range(L):
        pre = f"b{l}."
        h1, c1 = _ln(x, P[pre + "ln1.g"], P[pre + "ln1.b"])
        q = h1 @ P[pre + "q.W"] + P[pre + "q.b"]
        k = h1 @ P[pre + "k.W"] + P[pre + "k.b"]
        vv = h1 @ P[pre + "v.W"] + P[pre + "v.b"]
        att, probs = attention(q, k, vv, B, Ts, H)
        xm = x + att @ P[pre + "o.W"] + P[pre + "o.b"]
        h2, c2 = _ln(xm, P[pre + "ln2.g"], P[pre + "ln2.b"])
        f1 = np.maximum(h2 @ P[pre + "fc1.W"] + P[pre + "fc1.b"], 0.0)
        xo = xm + f1 @ P[pre + "fc2.W"] + P[pre + "fc2.b"]
        caches.append((x, h1, c1, q, k, vv, att, probs, xm, h2, c2, f1))
        x = xo
    hf, cf = _ln(x, P["lnf.g"], P["lnf.b"])
    logits = hf @ P["head.W"] + P["head.b"]
    z = logits - logits.max(1, keepdims=True)
    e = np.exp(z)
    p = e / e.sum(1, keepdims=True)
    y = targets.reshape(N).astype(np.int64)
    loss = -np.log(p[np.arange(N), y]).sum()
    dlog = p.copy()
    dlog[np.arange(N), y] -= 1.0
    dlog /= N
    G = {name: np.zeros(shape) for name, shape in layout(V, D, L, T, F)}
    G["head.W"] = hf.T @ dlog
    G["head.b"] = dlog.sum(0)
    dhf = dlog @ P["head.W"].T
    g, G["lnf.g"], G["lnf.b"] = _ln_bwd(dhf, P["lnf.g"], cf)
    for l in range(L - 1, -1, -1):
        pre = f"b{l}."
        (xin, h1, c1, q, k, vv, att, probs, xm, h2, c2, f1) = caches[l]
        G[pre + "fc2.W"] = f1.T @ g
        G[pre + "fc2.b"] = g.sum(0)
        df1 = (g @ P[pre + "fc2.W"].T) * (f1 > 0)
        G[pre + "fc1.W"] = h2.T @ df1
        G[pre + "fc1.b"] = df1.sum(0)
        dh2 = df1 @ P[pre + "fc1.W"].T
        dx2, G[pre + "ln2.g"], G[pre + "ln2.b"] = _ln_bwd(dh2, P[pre + "ln2.g"], c2)
        gm = g + dx2
        G[pre + "o.W"] = att.T @ gm
        G[pre + "o.b"] = gm.sum(0)
        datt = gm @ P[pre + "o.W"].T
        dq, dk, dv = attention_bwd(datt, q, k, vv, probs, B, Ts, H)
        dh1 = np.zeros_like(h1)
        for name, dd in (("q", dq), ("k", dk), ("v", dv)):
            G[pre + name + ".W"] = h1.T @ dd
            G[pre + name + ".b"] = dd.sum(0)
            dh1 += dd @ P[pre + name + ".W"].T
        dx1, G[pre + "ln1.g"], G[pre + "ln1.b"] = _ln_bwd(dh1, P[pre + "ln1.g"], c1)
        g = gm + dx1
    np.add.at(G["tok"], ids, g)
    np.add.at(G["pos"], pos, g)
    grads = flatten(G, V, D, L, T, F)
    w = np.asarray(flat, np.float64)
    if opt == "adam":
        b1, b2, eps = betas
        m = np.zeros_like(w) if m is None else m
        v = np.zeros_like(w) if v is None else v
        m = b1 * m + (1 - b1) * grads
        v = b2 * v + (1 - b2) * grads ** 2
        new = w - lr * (m / (1 - b1 ** t)) / (np.sqrt(v / (1 - b2 ** t)) + eps)
    elif opt == "sgd":
        new = w - lr * grads
    else:
        new = w
    return loss, grads, new, m, v, logits


def attention_cached(q, k, v, H):
    """MultiHeadAttention::attendHeadCached per head (src/Attention/MultiHeadAttention.php:127-137),
    heads concatenated: q [n, D] new rows, k, v [len, D] all cached rows; softmax of
    (q k^T) / sqrt(head_dim) over every cached key -- no mask."""
    D = q.shape[1]
    dh = D // H
    scale = 1.0 / np.sqrt(dh)
    outs = []
    for h in range(H):
        cs = slice(h * dh, (h + 1) * dh)
        s = q[:, cs] @ k[:, cs].T * scale
        s = s - s.max(1, keepdims=True)
        e = np.exp(s)
        outs.append((e / e.sum(1, keepdims=True)) @ v[:, cs])
    return np.concatenate(outs, 1)


def forward_cached(flat, tokens, cache, V, D, H, L, T, F):
    """TransformerLM::forwardWithCache (src/Transformers/TransformerLM.php:124-151)
    in float64.  tokens: [n] ints for positions cache['len'] .. cache['len']+n-1;
    cache: {'len': int, 'k': [L arrays [len, D]], 'v': [...]} (KVCache), updated
    in place.  Per block (TransformerBlock.php:40-45): x += attn(ln1(x)) with the
    new K/V rows appended to the layer's cache (MultiHeadAttention.php:99-125)
    and every query row attending to ALL cached keys -- attendHeadCached
    (MultiHeadAttention.php:127-137) applies no causal mask -- then
    x += ffn(ln2(x)).  Returns logits [n, V]."""
    n = len(tokens)
    off = cache["len"]
    if off + n > T:
        raise RuntimeError(f"Sequence position {off + n} exceeds max {T}.")
    P = unflatten(np.asarray(flat, np.float64), V, D, L, T, F)
    ids = np.asarray(tokens, np.int64)
    x = P["tok"][ids] + P["pos"][off:off + n]
    for l in range(L):
        pre = f"b{l}."
        h1, _ = _ln(x, P[pre + "ln1.g"], P[pre + "ln1.b"])
        q = h1 @ P[pre + "q.W"] + P[pre + "q.b"]
        k = h1 @ P[pre + "k.W"] + P[pre + "k.b"]
        vv = h1 @ P[pre + "v.W"] + P[pre + "v.b"]
        if off:
            k = np.concatenate([cache["k"][l], k])
            vv = np.concatenate([cache["v"][l], vv])
        if len(cache["k"]) <= l:
            cache["k"].append(k)
            cache["v"].append(vv)
        else:
            cache["k"][l], cache["v"][l] = k, vv
        x = x + attention_cached(q, k, vv, H) @ P[pre + "o.W"] + P[pre + "o.b"]
        h2, _ = _ln(x, P[pre + "ln2.g"], P[pre + "ln2.b"])
        f1 = np.maximum(h2 @ P[pre + "fc1.W"] + P[pre + "fc1.b"], 0.0)
        x = x + f1 @ P[pre + "fc2.W"] + P[pre + "fc2.b"]
    cache["len"] = off + n
    hf, _ = _ln(x, P["lnf.g"], P["lnf.b"])
    return hf @ P["head.W"] + P["head.b"]


def new_cache():
    """TransformerLM::newCache (src/Transformers/TransformerLM.php:153-156)."""
    return {"len": 0, "k": [], "v": []}
