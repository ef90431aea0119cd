"""Staged host steps (zilla_net_stage_host / zilla_net_step_staged, GPU).

The next batch's host->device copy runs on a copy stream during the current
step; the arithmetic is the step's own, so N staged steps must leave the
parameters and losses bit-identical to N zilla_net_step_host steps on the same
batches.  Also the slot rules: stepping with nothing staged and staging a third
batch before a step are rejected with -2.
"""
import numpy as np
import pytest

from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import Net

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,precision,batch", [("large_cnn", 1, 128), ("cnn_1x8_pool_fc", 0, 64)])
def test_staged_steps_match_host_steps(name, precision, batch):
    w = configs.WORKLOADS[name]
    p0 = synthetic.init_params(w, seed=5)
    batches = [synthetic.batch(w, batch, seed=5, step=s) for s in range(3)]
    a = Net(w, batch=batch, precision=precision)
    b = Net(w, batch=batch, precision=precision)
    try:
        a.set_params(p0)
        b.set_params(p0)
        la = [a.step_host(x, y) for x, y in batches]
        b.stage_host(*batches[0])
        lb = []
        for s in range(3):
            if s + 1 < 3:
                b.stage_host(*batches[s + 1])
            lb.append(b.step_staged())
        a.device_status()
        b.device_status()
        assert la == lb, (la, lb)
        assert np.array_equal(a.params(), b.params()), "staged steps diverged from host steps"
    finally:
        a.close()
        b.close()


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
