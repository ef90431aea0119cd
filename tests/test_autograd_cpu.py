"""The batched autograd bridge (zillaphp_b200.autograd) on the CPU: its graph
wiring, gradient accumulation, broadcasting and optimizer bookkeeping, with
every device op computed by the oracle (tests/oracle_backend.py).  One
Trainer step per batch must reproduce the oracle's replay of the reference
step sequence (oracle.StepModel) on the same weights and inputs: loss x batch
equal to the step's loss sum (relative 1e-6), gradients and updated weights
normwise 1e-6 (both sides run the same oracle ops; only the graph order can
differ), and the first step's pool argmax equal."""
import numpy as np
import pytest

import npref
import oracle
import oracle_backend
from zillaphp_b200 import autograd as ag
from zillaphp_b200 import configs, synthetic


@pytest.fixture()
def fake():
    prev = ag._BACKEND
    ag.release_pool()
    ag._BACKEND = oracle_backend.OracleBackend()
    ag._POOL = ag._Pool()
    yield ag._BACKEND
    ag._BACKEND = prev
    ag._POOL = ag._Pool()


def make(w, flat):
    model = ag.sequential_from_spec(w.layers, w.in_shape)
    model.load_flat(flat)
    params = model.parameters()
    if w.optimizer == configs.ADAM:
        b1, b2, eps = w.adam
        opt = ag.Adam(params, w.lr, b1, b2, eps)
    else:
        opt = ag.SGD(params, w.lr)
    return model, ag.Trainer(model, opt, ag.CrossEntropy())


@pytest.mark.parametrize("name,batch", [("mlp_784_128_10", 8), ("cnn_1x8_pool_fc", 6), ("large_cnn", 2),
                                        ("audio_kws_cnn", 2)])
def test_bridge_steps_match_oracle_step(fake, name, batch):
    w = configs.WORKLOADS[name]
    p0 = synthetic.init_params(w, seed=21)
    ref = oracle.StepModel(w.spec(), batch, w.in_shape, kind="oracle")
    ref.params[:] = p0
    model, trainer = make(w, p0)
    for step in range(2):
        x, y = synthetic.batch(w, batch, seed=21, step=step)
        x4 = x.reshape((batch,) + tuple(w.in_shape))
        rl = ref.step(x, y, opt=w.optimizer, lr=w.lr)
        bl = trainer.step(x4, y)
        # the step sequence's loss is softmax_ce_dev's (no clamp); CrossEntropy clamps p_t at
        # 1e-12 (CrossEntropy.php:58), so where a row falls below it the bar is that loss
        z = ref.output(len(w.layers) - 1, batch * w.classes).reshape(batch, w.classes).astype(np.float64)
        pz = np.exp(z - z.max(1, keepdims=True))
        pt = (pz / pz.sum(1, keepdims=True))[np.arange(batch), y.astype(np.int64)]
        if (pt < 1e-12).any():   # CrossEntropy's loss (float64, as the PHP class) from the same logits
            rl = float(-np.log(np.maximum(pt, 1e-12)).sum())
        assert abs(bl * batch - rl) <= 1e-6 * abs(rl), (step, bl * batch, rl)
        assert npref.normwise(model.flat(grads=True), ref.grads) < 1e-6
        assert npref.normwise(model.flat(), ref.params) < 1e-6


def test_bridge_pool_argmax_and_calls(fake):
    w, batch = configs.CNN_SMALL, 4
    p0 = synthetic.init_params(w, seed=5)
    ref = oracle.StepModel(w.spec(), batch, w.in_shape, kind="oracle")
    ref.params[:] = p0
    model, trainer = make(w, p0)
    x, y = synthetic.batch(w, batch, seed=5)
    ref.step(x, y, opt=0, lr=0.0)
    pooled = model.layers[0](ag.Tensor.from_numpy(x.reshape(batch, 1, 28, 28)))
    pooled = model.layers[2](model.layers[1](pooled))
    n = batch * 8 * 13 * 13
    got = pooled.argmax.numpy().ravel().view(np.int32).reshape(batch, -1) % (26 * 26)
    assert np.array_equal(got.ravel(), ref.argmax(2, n))
    fake.calls.clear()
    trainer.step(x.reshape(batch, 1, 28, 28), y)
    assert fake.calls == ["conv2d_batched_fwd_dev", "maxpool2d_batched_fwd_dev", "maxpool2d_batched_bwd_dev",
                          "conv2d_batched_bwd_dev"]


def test_gradient_accumulates_over_two_uses(fake):
    """A tensor used twice receives the sum of both gradients (accumulateGrad)."""
    W = ag.Parameter(np.arange(6, dtype=np.float32).reshape(2, 3) / 10)
    x = ag.Tensor.from_numpy(np.ones((4, 2), np.float32))
    z = x.matmul(W)
    s = z.add(z)                                  # the same tensor on both sides
    loss = ag.CrossEntropy().forward(s, [0, 1, 2, 0])
    loss.backward()
    zn = 2 * (np.ones((4, 2)) @ (np.arange(6).reshape(2, 3) / 10))
    p = np.exp(zn - zn.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    g = p.copy()
    g[np.arange(4), [0, 1, 2, 0]] -= 1
    g /= 4
    np.testing.assert_allclose(W.grad.numpy(), np.ones((4, 2)).T @ (2 * g), atol=1e-6)
    np.testing.assert_allclose(loss.item(), -np.log(p[np.arange(4), [0, 1, 2, 0]]).mean(), rtol=1e-6)


def test_scaled_loss_scales_the_gradient(fake):
    """loss.mul(k) before backward(): CrossEntropy's backward multiplies by the upstream
    gradient g->item() (src/Loss/CrossEntropy.php:69-70), so every gradient scales by k."""
    g = np.random.default_rng(3)
    Wn = g.standard_normal((5, 4)).astype(np.float32)
    xn = g.standard_normal((6, 5)).astype(np.float32)
    t = [0, 1, 2, 3, 1, 0]
    grads = []
    for k in (1.0, 0.5, -3.0):
        W = ag.Parameter(Wn)
        z = ag.Tensor.from_numpy(xn).matmul(W)
        loss = ag.CrossEntropy().forward(z, t)
        root = loss if k == 1.0 else loss.mul(ag.Tensor.from_numpy(np.array([k], np.float32)))
        root.backward()
        grads.append(W.grad.numpy().copy())
        if k != 1.0:
            np.testing.assert_allclose(root.item(), k * loss.item(), rtol=1e-6)
    np.testing.assert_allclose(grads[1], 0.5 * grads[0], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(grads[2], -3.0 * grads[0], rtol=1e-6, atol=1e-7)


def test_cross_entropy_clamps_the_target_probability(fake):
    """CrossEntropy.php:58 takes -log(max(p, 1e-12)): a row whose target logit trails by 100
    (p_t ~ 4e-44) adds 27.631 to the sum, not 100; the gradient is unclamped (p - onehot) / B."""
    zn = np.array([[0.0, 100.0, 0.0], [1.0, 2.0, 3.0]], np.float32)
    t = [0, 2]
    z = ag.Parameter(zn)
    loss = ag.CrossEntropy().forward(z, t)
    loss.backward()
    zz = zn.astype(np.float64)
    p = np.exp(zz - zz.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    want = -np.log(np.maximum(p[np.arange(2), t], 1e-12)).mean()
    np.testing.assert_allclose(loss.item(), want, rtol=1e-6)
    assert abs(loss.item() - (-np.log(1e-12) - np.log(p[1, 2])) / 2) < 1e-4
    g = p.copy()
    g[np.arange(2), t] -= 1
    np.testing.assert_allclose(z.grad.numpy(), g / 2, atol=1e-7)


def test_no_grad_records_nothing(fake):
    W = ag.Parameter(np.ones((3, 2), np.float32))
    with ag.no_grad():
        z = ag.Tensor.from_numpy(np.ones((1, 3), np.float32)).matmul(W)
    assert not z.requires_grad and z.backward_fn is None
    np.testing.assert_array_equal(z.numpy(), [[3.0, 3.0]])


def test_buffers_are_recycled(fake):
    model, trainer = make(configs.CNN_SMALL, synthetic.init_params(configs.CNN_SMALL, seed=1))
    x, y = synthetic.batch(configs.CNN_SMALL, 4, seed=1)
    trainer.step(x.reshape(4, 1, 28, 28), y)
    live = len(fake.bufs)
    for _ in range(3):
        trainer.step(x.reshape(4, 1, 28, 28), y)
    assert len(fake.bufs) == live      # steady state: every temporary comes from the pool


def test_buffer_returns_to_its_own_pool(fake):
    """A tensor freed after the pool was replaced (another backend) does not
    hand its handle to the new pool."""
    t = ag.Tensor.from_numpy(np.ones(7, np.float32))
    old = ag._POOL
    ag._POOL = ag._Pool()
    del t
    assert old.free.get(7) and not ag._POOL.free
