"""The Transformer-LM step with its Linear layers on TF32 tensor cores
(zilla_lm_set_precision(net, 1), GPU), at the config's 64 x 128 tokens and at
a second shape (32 x 64).

The Q/K/V, output and FFN projections and their input and weight gradients
run as tcgen05 kind::tf32 GEMMs, and so does the attention (S = Q K^T, O = P V
and the backward's five products, one CTA per sequence and head): the fp32
operands are read with a 10-bit mantissa (relative rounding 2^-11) and
accumulated in fp32.  The softmax, LayerNorm, the head, the loss and Adam run
in fp32 on CUDA cores.  Tolerances against the float64 oracle restatement
(oracle/lm_oracle.py), stated for TF32, with the values measured on a B200 in
brackets (64 x 128, 32 x 64):
  loss sum            relative 2e-4   [2.1e-5, 1.3e-5]
  gradients           normwise 2e-2 over the whole flat buffer [5.9e-3, 1.1e-2]
  three-step losses   relative 2e-4 against the oracle's own trajectory and
                      against the fp32 engine's [2.4e-5]
The 32 x 64 shape runs the attention with a short tile: rows 64..127 of each
128-row tile belong to the next sequence (or lie past the batch) and must add
nothing.
"""
import numpy as np
import pytest

import lm_oracle
import npref
from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import LM

pytestmark = pytest.mark.gpu
W = configs.TRANSFORMER_LM


def oracle_step(flat, tok, tgt, batch, seq, **kw):
    return lm_oracle.step(flat, tok.reshape(batch, seq).astype(np.int64), tgt.reshape(batch, seq).astype(np.int64),
                          W.vocab, W.dim, W.heads, W.layers, W.max_seq, W.ffn, **kw)


@pytest.mark.parametrize("batch,seq", [(64, 128), (32, 64)])
def test_tf32_step_against_oracle(batch, seq):
    p0 = synthetic.lm_init_params(W, seed=7, perturb=0.1)
    tok, tgt = synthetic.lm_batch(W, batch, seq, seed=7)
    net = LM(W, batch=batch, seq=seq, precision=1)
    try:
        net.set_params(p0)
        loss = net.step_host(tok, tgt, update=False)
        net.device_status()
        g = net.grads()
    finally:
        net.close()
    rl, rg, *_ = oracle_step(p0.astype(np.float64), tok, tgt, batch, seq, opt="none")
    lerr = abs(loss - rl) / abs(rl)
    gerr = npref.normwise(g, rg)
    print(f"tf32 LM {batch}x{seq}: loss rel {lerr:.2e}, gradients normwise {gerr:.2e}")
    assert lerr < 2e-4, (loss, rl)
    assert gerr < 2e-2


def test_tf32_trajectory_and_fp32_agreement():
    batch, seq = 64, 128
    p0 = synthetic.lm_init_params(W, seed=9, perturb=0.1)
    nets = [LM(W, batch=batch, seq=seq, precision=p) for p in (0, 1)]
    flat = p0.astype(np.float64)
    m = v = None
    worst, worst32 = 0.0, 0.0
    try:
        for n in nets:
            n.set_params(p0)
        for k in range(3):
            tok, tgt = synthetic.lm_batch(W, batch, seq, seed=9, step=k)
            l32, l16 = (n.step_host(tok, tgt, update=True) for n in nets)
            rl, _, flat, m, v, _ = oracle_step(flat, tok, tgt, batch, seq, opt="adam", lr=W.lr, t=k + 1, m=m, v=v)
            worst = max(worst, abs(l16 - rl) / abs(rl))
            worst32 = max(worst32, abs(l16 - l32) / abs(l32))
            print(f"step {k}: oracle {rl:.4f} fp32 {l32:.4f} tf32 {l16:.4f}")
        for n in nets:
            n.device_status()
    finally:
        for n in nets:
            n.close()
    print(f"tf32 trajectory: worst loss gap to the oracle {worst:.2e}, to the fp32 engine {worst32:.2e}")
    assert worst < 2e-4
    assert worst32 < 2e-4
