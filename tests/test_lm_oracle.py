"""Pins the Transformer-LM oracle (CPU).

1. Parameter layout: 429,889 parameters at the BASELINE configuration
   (vocab 65, d 128, 4 heads, 2 blocks, FFN 512, 128 positions).
2. Attention against the reference's full-attention known-answer test
   (tests/golden/reference_kat.json "attention_full").
3. The hand-written backward against central finite differences (the
   reference's own gradient-check strategy, tests/Numerical/GradientCheckTest.php),
   on a small model in float64.
"""
import numpy as np

import lm_oracle


def test_layout_size():
    n = sum(int(np.prod(s)) for _, s in lm_oracle.layout(65, 128, 2, 128, 512))
    assert n == 429_889


def test_layout_matches_library_layout():
    from zillaphp_b200 import configs, synthetic
    w = configs.TRANSFORMER_LM
    assert synthetic.lm_layout(w) == lm_oracle.layout(w.vocab, w.dim, w.layers, w.max_seq, w.ffn)


def test_attention_kat(golden):
    g = golden["attention_full"]
    N, D = g["N"], g["D"]
    q = np.array(g["Q"]).reshape(N, D)
    k = np.array(g["K"]).reshape(N, D)
    v = np.array(g["V"]).reshape(N, D)
    out, _ = lm_oracle.attention(q, k, v, 1, N, 1)
    np.testing.assert_allclose(out.ravel(), g["expected"], atol=g["tol"])


def test_backward_matches_finite_differences():
    V, D, H, L, T, F, B, Ts = 7, 8, 2, 2, 6, 12, 2, 5
    rng = np.random.default_rng(0)
    n = sum(int(np.prod(s)) for _, s in lm_oracle.layout(V, D, L, T, F))
    flat = rng.standard_normal(n) * 0.3
    tokens = rng.integers(0, V, (B, Ts))
    targets = rng.integers(0, V, (B, Ts))
    loss, grads, *_ = lm_oracle.step(flat, tokens, targets, V, D, H, L, T, F, opt="none")
    idx = rng.choice(n, 60, replace=False)
    eps = 1e-6
    for i in idx:
        fp, fm = flat.copy(), flat.copy()
        fp[i] += eps
        fm[i] -= eps
        lp = lm_oracle.step(fp, tokens, targets, V, D, H, L, T, F, opt="none")[0]
        lmn = lm_oracle.step(fm, tokens, targets, V, D, H, L, T, F, opt="none")[0]
        num = (lp - lmn) / (2 * eps) / (B * Ts)     # loss is a sum; gradients are of the mean
        assert abs(num - grads[i]) <= 1e-6 + 1e-5 * abs(num), (i, num, grads[i])
