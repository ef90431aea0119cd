"""The fused training step (zilla_net_step, one C call per step) against the
oracle's replay of the reference step sequence (GPU).

fp32 engine (precision 0): forward contractions follow the reference order,
so the first step's pool argmax must be bit-identical; losses, gradients
and updated weights within 1e-4 normwise over three steps (SGD or Adam).
"""
import numpy as np
import pytest

import npref
import oracle
from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import Net

pytestmark = pytest.mark.gpu

CASES = [("mlp_784_128_10", 64), ("cnn_1x8_pool_fc", 64), ("large_cnn", 4), ("audio_kws_cnn", 3)]


def channel_local(global_arg, B, C, H, W):
    """GPU batched argmax (flat into [B,C,H,W]) -> CPU convention (ih*W + iw)."""
    return (global_arg.reshape(B, -1) % (H * W)).ravel()


@pytest.mark.parametrize("name,batch", CASES)
def test_fp32_step_matches_oracle(name, batch):
    w = configs.WORKLOADS[name]
    p0 = synthetic.init_params(w, seed=11)
    ref = oracle.StepModel(w.spec(), batch, w.in_shape, kind="oracle")
    ref.params[:] = p0
    net = Net(w, batch=batch, precision=0)
    net.set_params(p0)
    for step in range(3):
        x, y = synthetic.batch(w, batch, seed=11, step=step)
        rl = ref.step(x, y, opt=w.optimizer, lr=w.lr)
        gl = net.step_host(x, y)
        assert abs(gl - rl) / abs(rl) < 1e-5, (step, gl, rl)
        assert npref.normwise(net.grads(), ref.grads) < 1e-4
        assert npref.normwise(net.params(), ref.params) < 1e-4
        if step == 0:
            # pool argmax bit-exact (same forward bits on both sides)
            shape = (1,) + tuple(w.in_shape)
            c, h, wd = w.in_shape
            for li, (kind, a, b, pad) in enumerate(w.layers):
                if kind == configs.CONV:
                    c, h, wd = b, h + 2 * pad - 2, wd + 2 * pad - 2
                elif kind == configs.POOL:
                    oh, ow = (h - 2) // 2 + 1, (wd - 2) // 2 + 1
                    n = batch * c * oh * ow
                    got = channel_local(net.argmax(li, n), batch, c, h, wd)
                    assert np.array_equal(got, ref.argmax(li, n)), f"layer {li}"
                    h, wd = oh, ow
            del shape
    net.close()


def test_fp32_step_device_resident_inputs():
    """zilla_net_step on registry handles equals zilla_net_step_host."""
    from zillaphp_b200.backend import B200Backend
    be = B200Backend()
    w = configs.CNN_SMALL
    p0 = synthetic.init_params(w, seed=2)
    x, y = synthetic.batch(w, 64, seed=2)
    a, b = Net(w, precision=0), Net(w, precision=0)
    a.set_params(p0); b.set_params(p0)
    ix, iy, il = be.bufferAlloc(x.size), be.bufferAlloc(64), be.bufferAlloc(1)
    be.bufferUpload(ix, x); be.bufferUpload(iy, y)
    a.step_dev(ix, iy, il)
    lb = b.step_host(x, y)
    assert be.bufferDownload(il, 1)[0] == lb
    assert np.array_equal(a.params(), b.params())
