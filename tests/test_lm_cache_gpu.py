"""Generation with a K/V cache (zilla_lm_forward_cached, TransformerLM::forwardWithCache)
against the float64 oracle (oracle/lm_oracle.py forward_cached) on the GPU.

Each call is compared with the oracle's call on the same cache state:
logits max |err| <= 1e-4 of the largest |logit| (fp32 device arithmetic
against float64).  The sequence follows Sampler::generate: a prompt in one
call (attention without a mask), then one token per call, a reset and a new
prompt (the sliding window), up to the max_seq positions.
"""
import numpy as np
import pytest

import lm_oracle
from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import LM

pytestmark = pytest.mark.gpu

W = configs.TRANSFORMER_LM
DIMS = (W.vocab, W.dim, W.heads, W.layers, W.max_seq, W.ffn)


def close(got, ref):
    err = float(np.max(np.abs(got - ref)) / np.max(np.abs(ref)))
    assert err < 1e-4, err


@pytest.fixture(scope="module")
def model():
    p0 = synthetic.lm_init_params(W, seed=11, perturb=0.1)
    net = LM(W, batch=2, seq=16)
    net.set_params(p0)
    yield net, p0.astype(np.float64)
    net.close()


def test_prompt_then_tokens(model):
    net, flat = model
    rng = np.random.default_rng(3)
    net.cache_reset()
    cache = lm_oracle.new_cache()
    prompt = rng.integers(0, W.vocab, 20)
    close(net.forward_cached(prompt), lm_oracle.forward_cached(flat, prompt, cache, *DIMS))
    for _ in range(12):
        t = rng.integers(0, W.vocab, 1)
        got = net.forward_cached(t)
        assert got.shape == (1, W.vocab)
        close(got, lm_oracle.forward_cached(flat, t, cache, *DIMS))
    assert net.cache_length() == cache["len"] == 32


def test_fill_to_max_seq_overflow_and_reset(model):
    net, flat = model
    rng = np.random.default_rng(4)
    net.cache_reset()
    cache = lm_oracle.new_cache()
    prompt = rng.integers(0, W.vocab, W.max_seq - 3)
    close(net.forward_cached(prompt), lm_oracle.forward_cached(flat, prompt, cache, *DIMS))
    for _ in range(3):
        t = rng.integers(0, W.vocab, 1)
        close(net.forward_cached(t), lm_oracle.forward_cached(flat, t, cache, *DIMS))
    assert net.cache_length() == W.max_seq
    with pytest.raises(RuntimeError, match="exceeds max"):
        net.forward_cached([1])
    assert net.cache_length() == W.max_seq           # unchanged by the failed call
    net.cache_reset()                                 # Sampler's sliding window: new cache, re-prompt
    assert net.cache_length() == 0
    full = rng.integers(0, W.vocab, W.max_seq)        # the largest single call
    close(net.forward_cached(full), lm_oracle.forward_cached(flat, full, lm_oracle.new_cache(), *DIMS))


def test_token_ids_follow_embedding_cast(model):
    net, flat = model
    net.cache_reset()
    for bad in ([W.vocab], [-1.5], [np.nan]):
        with pytest.raises(RuntimeError, match="out of range"):
            net.forward_cached(bad)
        assert net.cache_length() == 0
    got = net.forward_cached([W.vocab - 0.3, 0.7])    # (int) truncates: ids vocab-1 and 0
    close(got, lm_oracle.forward_cached(flat, [W.vocab - 1, 0], lm_oracle.new_cache(), *DIMS))


def test_generation_uses_trained_parameters():
    p0 = synthetic.lm_init_params(W, seed=12, perturb=0.1)
    net = LM(W, batch=2, seq=16)
    net.set_params(p0)
    tok, tgt = synthetic.lm_batch(W, 2, 16, seed=12)
    net.step_host(tok, tgt, update=True)
    flat = net.params().astype(np.float64)
    prompt = tok[:16].astype(np.int64)
    cache = lm_oracle.new_cache()
    close(net.forward_cached(prompt), lm_oracle.forward_cached(flat, prompt, cache, *DIMS))
    close(net.forward_cached([5]), lm_oracle.forward_cached(flat, [5], cache, *DIMS))
    net.device_status()
    net.close()
