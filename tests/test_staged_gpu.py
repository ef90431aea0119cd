"""Staged host steps (zilla_net_stage_host / zilla_net_step_staged /
zilla_net_step_staged_deferred, GPU).

The next batch's host->device copy runs on a copy stream during the current
step; the arithmetic is the step's own, so N staged steps must leave the
parameters and losses bit-identical to N zilla_net_step_host steps on the same
batches, and the deferred variant (each call hands out the previous step's
loss) must give the same losses in the same order.  The staged runs are also
held against the oracle's replay of the reference step sequence: the fp32
engine within 1e-5 (losses) and 1e-4 (weights, normwise), the bf16 engine on
its first step's loss within 1e-3.  Also the slot rules: stepping with nothing
staged and staging a third batch before a step are rejected with -2.
"""
import os

import numpy as np
import pytest

import npref
import oracle
from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import Net

pytestmark = pytest.mark.gpu


def _oracle_run(w, batch, p0, batches):
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else 1
    ref = oracle.StepModel(w.spec(), batch, w.in_shape, nthreads=threads)
    ref.params[:] = p0
    losses = [ref.step(x, y, w.optimizer, w.lr) for x, y in batches]
    return losses, ref.params.copy()


@pytest.mark.parametrize("name,precision,batch", [("large_cnn", 1, 128), ("cnn_1x8_pool_fc", 0, 64)])
def test_staged_steps_match_host_steps(name, precision, batch):
    w = configs.WORKLOADS[name]
    p0 = synthetic.init_params(w, seed=5)
    batches = [synthetic.batch(w, batch, seed=5, step=s) for s in range(3)]
    a = Net(w, batch=batch, precision=precision)
    b = Net(w, batch=batch, precision=precision)
    c = Net(w, batch=batch, precision=precision)
    try:
        for n in (a, b, c):
            n.set_params(p0)
        la = [a.step_host(x, y) for x, y in batches]
        b.stage_host(*batches[0])
        c.stage_host(*batches[0])
        lb, lc = [], []
        for s in range(3):
            if s + 1 < 3:
                b.stage_host(*batches[s + 1])
                c.stage_host(*batches[s + 1])
            lb.append(b.step_staged())
            prev = c.step_staged_deferred()
            assert (prev is None) == (s == 0)
            if prev is not None:
                lc.append(prev)
        lc.append(c.loss_flush())
        assert c.loss_flush() is None
        for n in (a, b, c):
            n.device_status()
        assert la == lb, (la, lb)
        assert lb == lc, (lb, lc)
        assert np.array_equal(a.params(), b.params()), "staged steps diverged from host steps"
        assert np.array_equal(b.params(), c.params()), "deferred staged steps diverged"
        rl, rp = _oracle_run(w, batch, p0, batches)
        if precision == 0:
            assert all(abs(g - r) <= 1e-5 * abs(r) for g, r in zip(lb, rl)), (lb, rl)
            assert npref.normwise(b.params(), rp) < 1e-4
        else:
            assert abs(lb[0] - rl[0]) <= 1e-3 * abs(rl[0]), (lb[0], rl[0])
    finally:
        a.close()
        b.close()
        c.close()


def test_staging_slot_rules():
    w = configs.WORKLOADS["cnn_1x8_pool_fc"]
    net = Net(w, batch=64, precision=0)
    try:
        net.set_params(synthetic.init_params(w, seed=6))
        x, y = synthetic.batch(w, 64, seed=6, step=0)
        with pytest.raises(RuntimeError):
            net.step_staged()          # nothing staged
        net.stage_host(x, y)
        net.stage_host(x, y)
        with pytest.raises(RuntimeError):
            net.stage_host(x, y)       # both slots hold batches not yet stepped
        net.step_staged()
        net.step_staged()
        net.device_status()
    finally:
        net.close()
