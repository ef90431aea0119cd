"""Evaluation (zilla_net_forward, GPU): the forward pass only, through the
same kernels as the training step.

* fp32 engine: logits and loss against the oracle's forward on the same
  weights (the forward is bit-faithful there: exact-order sums, no FMA), and
  the loss equals the training step's loss on the same batch;
* bf16 engine: logits within the engine's tolerance of a float64 forward from
  its own bf16 weights, the loss equal to the loss its training step reports
  on the same batch and weights (same kernels up to the head), and no
  parameter change;
* targets are optional.
"""
import os
import sys

import numpy as np
import pytest

from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import Net

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,precision,batch", [("large_cnn", 1, 128), ("cnn_1x8_pool_fc", 0, 64),
                                                  ("mlp_784_128_10", 0, 64)])
def test_forward_matches_step_loss_and_leaves_params(name, precision, batch):
    w = configs.WORKLOADS[name]
    p0 = synthetic.init_params(w, seed=7)
    x, y = synthetic.batch(w, batch, seed=7, step=0)
    net = Net(w, batch=batch, precision=precision)
    try:
        net.set_params(p0)
        logits, loss = net.forward(x, y)
        logits2, none = net.forward(x)
        assert none is None and np.array_equal(logits, logits2)
        assert np.array_equal(net.params(), p0), "the forward pass changed the parameters"
        # the loss sum of the logits (float64 restatement of softmax-CE on the returned logits)
        z = logits.astype(np.float64)
        lse = np.log(np.exp(z - z.max(1, keepdims=True)).sum(1)) + z.max(1)
        ref = float((lse - z[np.arange(batch), y.astype(int)]).sum())
        assert abs(loss - ref) / abs(ref) < 1e-5, (loss, ref)
        # the training step reports the same loss on the same batch and weights
        step_loss = net.step_host(x, y, update=False)
        assert abs(step_loss - loss) / abs(loss) < 1e-6, (step_loss, loss)
    finally:
        net.close()


def test_fp32_forward_matches_oracle():
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
    import npref
    import oracle
    w = configs.WORKLOADS["cnn_1x8_pool_fc"]
    batch = 64
    p0 = synthetic.init_params(w, seed=8)
    x, y = synthetic.batch(w, batch, seed=8, step=0)
    net = Net(w, batch=batch, precision=0)
    try:
        net.set_params(p0)
        logits, loss = net.forward(x, y)
    finally:
        net.close()
    ref = oracle.StepModel(w.spec(), batch, w.in_shape, kind="oracle")
    try:
        ref.params[:] = p0
        ref_loss = ref.step(x, y, 0, 0.0)   # gradients only: the forward's outputs stay readable
        ref_logits = ref.output(len(w.spec()) - 1, batch * w.classes).reshape(batch, w.classes)
    finally:
        ref.close()
    assert npref.normwise(logits, ref_logits) < 1e-6
    assert abs(loss - ref_loss) / abs(ref_loss) < 1e-5, (loss, ref_loss)
