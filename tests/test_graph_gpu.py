"""Per-step CUDA graphs (zilla_net_set_graph, GPU): capture on the second step
for an input set, replay afterwards with the optimizer's arguments of each step.
The replayed steps must leave parameters and losses bit-identical to plain
steps (SGD and Adam, fp32 and bf16 engines), keep doing so across an optimizer
change (which drops the graphs), and count their kernels as launches.  The
graph runs of the fp32 configs are also held against the oracle's replay of
the reference step sequence (losses within 1e-5, weights within 1e-4
normwise), with the same optimizer change at step 4.
"""
import os

import numpy as np
import pytest

import npref
import oracle
from zillaphp_b200 import configs, native, synthetic
from zillaphp_b200.net import LM, Net

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,precision,batch", [("mlp_784_128_10", 0, 64), ("cnn_1x8_pool_fc", 0, 64),
                                                  ("large_cnn", 1, 128)])
def test_graph_steps_match_plain_steps(name, precision, batch):
    w = configs.WORKLOADS[name]
    p0 = synthetic.init_params(w, seed=11)
    batches = [synthetic.batch(w, batch, seed=11, step=s) for s in range(2)]
    lib = native.load()
    a, b = Net(w, batch=batch, precision=precision), Net(w, batch=batch, precision=precision)
    try:
        a.set_params(p0)
        b.set_params(p0)
        b.set_graph(True)
        la, lb, na, nb = [], [], [], []
        for s in range(6):
            x, y = batches[s % 2]
            if s == 4:   # an optimizer change drops the captured graphs
                for n in (a, b):
                    n._check(lib.zilla_net_set_optimizer(n.id, w.optimizer, w.lr * 0.5, *w.adam))
            c0 = lib.zilla_launch_count()
            la.append(a.step_host(x, y))
            c1 = lib.zilla_launch_count()
            lb.append(b.step_host(x, y))
            c2 = lib.zilla_launch_count()
            na.append(c1 - c0)
            nb.append(c2 - c1)
        a.device_status()
        b.device_status()
        assert la == lb, (la, lb)
        assert np.array_equal(a.params(), b.params()), "graph replays diverged from plain steps"
        assert na == nb, (na, nb)
        if precision == 0:
            threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else 1
            ref = oracle.StepModel(w.spec(), batch, w.in_shape, nthreads=threads)
            ref.params[:] = p0
            rl = [ref.step(*batches[s % 2], w.optimizer, w.lr if s < 4 else w.lr * 0.5) for s in range(6)]
            assert all(abs(g - r) <= 1e-5 * abs(r) for g, r in zip(lb, rl)), (lb, rl)
            assert npref.normwise(b.params(), ref.params) < 1e-4
    finally:
        a.close()
        b.close()


@pytest.mark.parametrize("precision", [0, 1])
def test_lm_graph_steps_match_plain_steps(precision):
    """The language model's step replayed from a graph: losses, parameters and launch
    counts equal to plain steps over six steps of two alternating token batches."""
    w = configs.TRANSFORMER_LM
    batch, seq = 8, 64
    p0 = synthetic.lm_init_params(w, seed=13, perturb=0.1)
    batches = [synthetic.lm_batch(w, batch, seq, seed=13, step=s) for s in range(2)]
    lib = native.load()
    a, b = LM(w, batch=batch, seq=seq, precision=precision), LM(w, batch=batch, seq=seq, precision=precision)
    try:
        a.set_params(p0)
        b.set_params(p0)
        b.set_graph(True)
        la, lb, na, nb = [], [], [], []
        for s in range(6):
            tok, tgt = batches[s % 2]
            c0 = lib.zilla_launch_count()
            la.append(a.step_host(tok, tgt))
            c1 = lib.zilla_launch_count()
            lb.append(b.step_host(tok, tgt))
            c2 = lib.zilla_launch_count()
            na.append(c1 - c0)
            nb.append(c2 - c1)
        a.device_status()
        b.device_status()
        assert la == lb, (la, lb)
        assert np.array_equal(a.params(), b.params()), "graph replays diverged from plain steps"
        assert na == nb, (na, nb)
    finally:
        a.close()
        b.close()
