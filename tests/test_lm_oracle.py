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


# ---- generation (TransformerLM::forwardWithCache)
def _small_lm(seed, L=2):
    V, D, H, T, F = 11, 16, 2, 12, 24
    rng = np.random.default_rng(seed)
    n = sum(int(np.prod(s)) for _, s in lm_oracle.layout(V, D, L, T, F))
    return rng.standard_normal(n) * 0.3, (V, D, H, L, T, F), rng


def test_cached_attention_kat(golden):
    """attendHeadCached applies no mask; the reference's causal attention
    known answer pins its newest row, which sees every key either way (one head)."""
    g = golden["attention_full"]
    N, D = g["N"], g["D"]
    q = np.array(g["Q"]).reshape(N, D)
    k = np.array(g["K"]).reshape(N, D)
    v = np.array(g["V"]).reshape(N, D)
    last = lm_oracle.attention_cached(q[-1:], k, v, 1).ravel()
    np.testing.assert_allclose(last, np.array(g["expected"]).reshape(N, D)[-1], atol=g["tol"])


def test_cached_one_token_at_a_time_equals_causal_forward():
    """One new token per call attends to exactly the earlier positions and
    itself, so token-by-token generation reproduces the causal forward."""
    flat, (V, D, H, L, T, F), rng = _small_lm(1)
    toks = rng.integers(0, V, (1, 9))
    *_, logits = lm_oracle.step(flat, toks, toks, V, D, H, L, T, F, opt="none")
    cache = lm_oracle.new_cache()
    rows = [lm_oracle.forward_cached(flat, [int(t)], cache, V, D, H, L, T, F) for t in toks[0]]
    assert cache["len"] == 9
    np.testing.assert_allclose(np.concatenate(rows), logits, rtol=0, atol=1e-12)


def test_cached_prompt_then_tokens():
    """A prompt in one call attends without a mask (its last row still equals
    the causal forward's for one block); later single tokens continue the cache."""
    flat, (V, D, H, L, T, F), rng = _small_lm(2, L=1)
    toks = rng.integers(0, V, (1, 10))
    *_, causal = lm_oracle.step(flat, toks, toks, V, D, H, L, T, F, opt="none")
    cache = lm_oracle.new_cache()
    prompt = lm_oracle.forward_cached(flat, toks[0, :6], cache, V, D, H, L, T, F)
    np.testing.assert_allclose(prompt[-1], causal[5], atol=1e-12)
    assert not np.allclose(prompt[0], causal[0])      # row 0 saw the later prompt rows
    nxt = lm_oracle.forward_cached(flat, toks[0, 6:7], cache, V, D, H, L, T, F)
    np.testing.assert_allclose(nxt[0], causal[6], atol=1e-12)


def test_cached_overflow_raises_and_keeps_cache():
    flat, (V, D, H, L, T, F), rng = _small_lm(3)
    cache = lm_oracle.new_cache()
    lm_oracle.forward_cached(flat, [1] * 10, cache, V, D, H, L, T, F)
    try:
        lm_oracle.forward_cached(flat, [1] * 3, cache, V, D, H, L, T, F)
        raise AssertionError("no overflow error")
    except RuntimeError as e:
        assert "exceeds max" in str(e)
    assert cache["len"] == 10
