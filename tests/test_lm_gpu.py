"""The fused Transformer-LM step (zilla_lm_create + zilla_net_step, fp32)
against the float64 oracle restatement of TransformerLM training
(oracle/lm_oracle.py) on the same seeded tokens and weights (GPU).

Tolerances (fp32 device arithmetic against float64):
  loss sum            relative 1e-5
  gradients           1e-4 normwise over the whole flat buffer, 1e-3 per tensor
                      (a tensor's error is taken relative to its own largest
                      entry, floored at 1e-4 of the whole buffer's: the key-bias
                      gradient is analytically zero -- a bias on every key shifts
                      a score row by a constant, which softmax ignores -- so
                      both sides hold only rounding noise there)
  updated parameters  the oracle's Adam applied to the device's own gradients,
                      1e-6 absolute (the update kernel is checked apart from the
                      gradient error that Adam's sign-like first step amplifies)
  three-step losses   relative 1e-4 against the oracle's own trajectory
"""
import numpy as np
import pytest

import lm_oracle
import npref
from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import LM

pytestmark = pytest.mark.gpu

W = configs.TRANSFORMER_LM


def dims(w):
    return w.vocab, w.dim, w.heads, w.layers, w.max_seq, w.ffn


def oracle_step(w, flat, tok, tgt, batch, seq, **kw):
    V, D, H, L, T, F = dims(w)
    return lm_oracle.step(flat, tok.reshape(batch, seq).astype(np.int64), tgt.reshape(batch, seq).astype(np.int64),
                          V, D, H, L, T, F, **kw)


def per_tensor(w, got, ref):
    worst, off = ("", 0.0), 0
    floor = 1e-4 * np.max(np.abs(ref))
    for name, shape in synthetic.lm_layout(w):
        n = int(np.prod(shape))
        a, b = got[off:off + n], ref[off:off + n]
        off += n
        e = float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), floor))
        if e > worst[1]:
            worst = (name, e)
    return worst


@pytest.mark.parametrize("batch,seq,perturb", [(4, 32, 0.1), (3, 50, 0.1), (64, 128, 0.0)])
def test_lm_step_matches_oracle(batch, seq, perturb):
    p0 = synthetic.lm_init_params(W, seed=5, perturb=perturb)
    tok, tgt = synthetic.lm_batch(W, batch, seq, seed=5)
    net = LM(W, batch=batch, seq=seq)
    net.set_params(p0)
    loss = net.step_host(tok, tgt, update=True)
    net.device_status()
    rl, rg, _, _, _, _ = oracle_step(W, p0.astype(np.float64), tok, tgt, batch, seq, opt="none")
    assert abs(loss - rl) / rl < 1e-5, (loss, rl)
    g = net.grads().astype(np.float64)
    assert npref.normwise(g, rg) < 1e-4
    name, err = per_tensor(W, g, rg)
    assert err < 1e-3, (name, err)
    # Adam update from the device's own gradients
    b1, b2, eps = W.adam
    m = (1 - b1) * g
    v = (1 - b2) * g * g
    want = p0 - W.lr * (m / (1 - b1)) / (np.sqrt(v / (1 - b2)) + eps)
    np.testing.assert_allclose(net.params(), want, atol=1e-6, rtol=0)
    net.close()


def test_lm_three_steps_track_oracle():
    batch, seq = 8, 64
    p = synthetic.lm_init_params(W, seed=9, perturb=0.05).astype(np.float64)
    net = LM(W, batch=batch, seq=seq)
    net.set_params(p.astype(np.float32))
    m = v = None
    for step in range(3):
        tok, tgt = synthetic.lm_batch(W, batch, seq, seed=9, step=step)
        got = net.step_host(tok, tgt)
        rl, _, p, m, v, _ = oracle_step(W, p, tok, tgt, batch, seq, opt="adam", lr=W.lr, t=step + 1, m=m, v=v)
        assert abs(got - rl) / rl < 1e-4, (step, got, rl)
    net.device_status()
    net.close()


def test_lm_device_resident_step_equals_host_step():
    from zillaphp_b200.backend import B200Backend
    be = B200Backend()
    batch, seq = 2, 40
    p0 = synthetic.lm_init_params(W, seed=3)
    tok, tgt = synthetic.lm_batch(W, batch, seq, seed=3)
    a, b = LM(W, batch=batch, seq=seq), LM(W, batch=batch, seq=seq)
    a.set_params(p0)
    b.set_params(p0)
    ix, iy, il = be.bufferAlloc(tok.size), be.bufferAlloc(tgt.size), be.bufferAlloc(1)
    be.bufferUpload(ix, tok)
    be.bufferUpload(iy, tgt)
    a.step_dev(ix, iy, il)
    lb = b.step_host(tok, tgt)
    assert be.bufferDownload(il, 1)[0] == lb
    assert np.array_equal(a.params(), b.params())
    for i in (ix, iy, il):
        be.bufferFree(i)
    a.close()
    b.close()
