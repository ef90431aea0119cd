"""The batched autograd bridge (zillaphp_b200.autograd: Tensor, Sequential,
CrossEntropy, SGD/Adam, Trainer) on the device ops of libzilla_b200 against
the oracle's replay of the reference step sequence (GPU).

Per Trainer step: the bridge's mean loss x batch equals the step's loss sum
within 1e-5 relative (where a row's target probability falls below 1e-12, the
bar is CrossEntropy's clamped loss, computed in float64 from the sequence's
logits); gradients and updated weights within 1e-4 normwise
(fp32 device arithmetic); the first step's pool argmax equal after mapping the
batched index to the reference's channel-local one.
"""
import numpy as np
import pytest

import npref
import oracle
from zillaphp_b200 import autograd as ag
from zillaphp_b200 import configs, synthetic

pytestmark = pytest.mark.gpu


def make(w, flat):
    model = ag.sequential_from_spec(w.layers, w.in_shape)
    model.load_flat(flat)
    if w.optimizer == configs.ADAM:
        b1, b2, eps = w.adam
        opt = ag.Adam(model.parameters(), w.lr, b1, b2, eps)
    else:
        opt = ag.SGD(model.parameters(), w.lr)
    return model, ag.Trainer(model, opt, ag.CrossEntropy())


@pytest.mark.parametrize("name,batch", [("mlp_784_128_10", 64), ("cnn_1x8_pool_fc", 64), ("large_cnn", 4),
                                        ("audio_kws_cnn", 3)])
def test_bridge_trains_like_the_reference_sequence(name, batch):
    w = configs.WORKLOADS[name]
    p0 = synthetic.init_params(w, seed=31)
    ref = oracle.StepModel(w.spec(), batch, w.in_shape, kind="oracle")
    ref.params[:] = p0
    model, trainer = make(w, p0)
    for step in range(3):
        x, y = synthetic.batch(w, batch, seed=31, step=step)
        rl = ref.step(x, y, opt=w.optimizer, lr=w.lr)
        bl = trainer.step(x.reshape((batch,) + tuple(w.in_shape)), y)
        # the step sequence's loss is softmax_ce_dev's (no clamp); CrossEntropy clamps p_t at
        # 1e-12 (CrossEntropy.php:58), so where a row falls below it the bar is that loss
        z = ref.output(len(w.layers) - 1, batch * w.classes).reshape(batch, w.classes).astype(np.float64)
        pz = np.exp(z - z.max(1, keepdims=True))
        pt = (pz / pz.sum(1, keepdims=True))[np.arange(batch), y.astype(np.int64)]
        if (pt < 1e-12).any():   # CrossEntropy's loss (float64, as the PHP class) from the same logits
            rl = float(-np.log(np.maximum(pt, 1e-12)).sum())
        assert abs(bl * batch - rl) / abs(rl) < 1e-5, (step, bl * batch, rl)
        assert npref.normwise(model.flat(grads=True), ref.grads) < 1e-4
        assert npref.normwise(model.flat(), ref.params) < 1e-4
    ag.backend().sync()


def test_bridge_pool_argmax_bit_exact():
    w, batch = configs.CNN_SMALL, 64
    p0 = synthetic.init_params(w, seed=8)
    ref = oracle.StepModel(w.spec(), batch, w.in_shape, kind="oracle")
    ref.params[:] = p0
    model, _ = make(w, p0)
    x, y = synthetic.batch(w, batch, seed=8)
    ref.step(x, y, opt=0, lr=0.0)
    t = ag.Tensor.from_numpy(x.reshape(batch, 1, 28, 28))
    pooled = model.layers[2](model.layers[1](model.layers[0](t)))
    got = pooled.argmax.numpy().ravel().view(np.int32).reshape(batch, -1) % (26 * 26)
    assert np.array_equal(got.ravel(), ref.argmax(2, batch * 8 * 13 * 13))


def test_bridge_eval_matches_fused_forward():
    """Under no_grad the bridge's logits equal the fused engine's evaluation (1e-5)."""
    from zillaphp_b200.net import Net
    w, batch = configs.CNN_SMALL, 64
    p0 = synthetic.init_params(w, seed=9)
    x, y = synthetic.batch(w, batch, seed=9)
    model, _ = make(w, p0)
    with ag.no_grad():
        logits = model(ag.Tensor.from_numpy(x.reshape(batch, 1, 28, 28))).numpy()
    net = Net(w, batch=batch, precision=0)
    net.set_params(p0)
    fused, _ = net.forward(x)
    net.close()
    assert npref.normwise(logits, fused) < 1e-5


def test_scaled_loss_scales_the_gradient_on_device():
    """loss.mul(k).backward() on the device ops: CrossEntropy's backward multiplies
    (p - onehot) / B by the upstream gradient (src/Loss/CrossEntropy.php:69-70), so the
    MLP's gradients are k times those of loss.backward(), checked against the oracle's
    step gradients (1e-4 normwise, fp32 device arithmetic)."""
    w, batch = configs.MLP, 64
    p0 = synthetic.init_params(w, seed=8)
    x, y = synthetic.batch(w, batch, seed=8)
    ref = oracle.StepModel(w.spec(), batch, w.in_shape, kind="oracle")
    ref.params[:] = p0
    ref.step(x, y, opt=0, lr=0.0)
    for k in (0.5, -2.0):
        model = ag.sequential_from_spec(w.layers, w.in_shape)
        model.load_flat(p0)
        xin = ag.Tensor.from_numpy(x.reshape((batch,) + tuple(w.in_shape)))
        loss = ag.CrossEntropy().forward(model(xin), y)
        loss.mul(ag.Tensor.from_numpy(np.array([k], np.float32))).backward()
        assert npref.normwise(model.flat(grads=True), k * ref.grads) < 1e-4
