"""The bf16 tcgen05 engine (precision 1) against the CPU oracle (GPU), at batch
64 and at the per-rank batches the step is benchmarked at (1024 = 8192 over 8
GPUs, 2048 = over 4).

Tolerances (bf16 operands, fp32 accumulation and fp32 master weights), with
the values measured on a B200 in brackets:
  packed bf16 weights           exact (round-to-nearest of the fp32 master)
  activations per layer         normwise <= 2e-2            [2.7e-3 .. 6.1e-3]
  pool argmax agreement         > 99.5% (conv2), > 99.3% (conv3): codes vs the
                                oracle's channel-local argmax [99.75%, 99.59%]
  loss                          relative <= 1e-3            [2.4e-5 .. 1.6e-4]
  gradients per parameter block normwise <= 0.1 at batch 64 [3.4e-3 .. 7.6e-2],
                                <= 3e-2 at 1024 and 2048     [4.8e-3 .. 2.6e-2]
  weights after one Adam step   normwise <= 1e-2            [2.5e-3]
The gradient gap comes from ReLU-mask and max-pool decisions that bf16
rounding flips near ties (0.25% of conv2's pool windows, 0.4% of conv3's),
each moving one sample's contribution to another pixel.  From batch 1024 on,
every block except the first conv's is near 1e-2; the first conv's weight and
bias gradients stay at 2-2.6e-2 as the batch grows, because they sum
per-sample terms that largely cancel, so the flip noise and the gradient grow
alike.  The kernels themselves are checked to fp32 accumulation accuracy in
test_tc_kernels_gpu.py.  A five-step Adam loss trajectory at batch 1024
follows the fp32 engine's within 6e-2 [3.6e-2]: Adam's first update moves
every weight by lr times the sign of its gradient, so weights whose gradient
is within flip noise of zero move 2 lr apart, and the loss after that step is
sensitive to them.  The tensor-core path is also deterministic: two identical
steps give bit-identical gradients.
"""
import numpy as np
import pytest

import npref
import oracle
from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import Net

pytestmark = pytest.mark.gpu

B = 64
BATCHES = (64, 1024, 2048)
LOSS_TOL = 1e-3
GRAD_TOL = {64: 0.1, 1024: 3e-2, 2048: 3e-2}
ARGMAX_AGREE = {"conv2.code": 0.995, "conv3.code": 0.993}
TRAJ_TOL = 6e-2


def bf16_round(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


def nchw_to_nhwc(a, Bn, C, H, W):
    return a.reshape(Bn, C, H, W).transpose(0, 2, 3, 1).ravel()


def blocks(w):
    off, out = 0, []
    for li, (kind, a, b, _) in enumerate(w.layers):
        if kind == configs.CONV:
            out += [(f"L{li}.W", off, b * a * 9), (f"L{li}.b", off + b * a * 9, b)]
            off += b * a * 9 + b
        elif kind == configs.LINEAR:
            out += [(f"L{li}.W", off, a * b), (f"L{li}.b", off + a * b, b)]
            off += a * b + b
    return out


@pytest.fixture(scope="module", params=BATCHES, ids=[f"B{b}" for b in BATCHES])
def large_step(request):
    import os
    Bn = request.param
    w = configs.CNN_LARGE
    p0 = synthetic.init_params(w, seed=21)
    x, y = synthetic.batch(w, Bn, seed=21)
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    ref = oracle.StepModel(w.spec(), Bn, w.in_shape, nthreads=threads)
    ref.params[:] = p0
    rl = ref.step(x, y, w.optimizer, w.lr)
    net = Net(w, batch=Bn, precision=1)
    net.set_params(p0)
    gl = net.step_host(x, y)
    net.device_status()
    views = net.inspect()
    out = dict(B=Bn, w=w, p0=p0, x=x, y=y, ref=ref, rl=rl, net=net, gl=gl, views=views,
               grads=net.grads(), params=net.params())
    yield out
    net.close()


def test_packed_weights_exact(large_step):
    v, p0 = large_step["views"], large_step["p0"]
    W2 = p0[320:320 + 64 * 32 * 9].reshape(64, 32, 9)
    assert np.array_equal(v["conv2.wf"], bf16_round(W2.transpose(2, 0, 1)).ravel())        # [t][co][ci]
    assert np.array_equal(v["conv2.wd"], bf16_round(W2[:, :, ::-1].transpose(2, 1, 0)).ravel())  # [t][ci][co]


def test_forward_activations(large_step):
    s, ref, v, Bn = large_step, large_step["ref"], large_step["views"], large_step["B"]
    errs = {}
    # layer outputs of the oracle (NCHW fp32): 1 relu(conv1), 4 pool(conv2), 7 pool(conv3), 9 relu(fc1)
    c1 = nchw_to_nhwc(ref.output(1, Bn * 32 * 28 * 28), Bn, 32, 28, 28)
    errs["conv1"] = npref.normwise(v["conv1.out"], c1)
    p2 = nchw_to_nhwc(ref.output(4, Bn * 64 * 14 * 14), Bn, 64, 14, 14)
    errs["conv2"] = npref.normwise(v["conv2.out"], p2)
    p3 = nchw_to_nhwc(ref.output(7, Bn * 128 * 7 * 7), Bn, 128, 7, 7)
    errs["conv3"] = npref.normwise(v["conv3.out"], p3)
    errs["fc1"] = npref.normwise(v["hidden.out"], ref.output(9, Bn * 256))
    print(f"B={Bn} forward normwise errors:", errs)
    assert all(e < 2e-2 for e in errs.values()), errs
    # argmax agreement of the fused pool epilogues with the oracle (codes vs channel-local argmax)
    for layer, C, H, key in ((4, 64, 14, "conv2.code"), (7, 128, 7, "conv3.code")):
        am = ref.argmax(layer, Bn * C * H * H).reshape(Bn, C, H, H)
        oh = np.arange(H)[:, None]; ow = np.arange(H)[None, :]
        pos = (am // (2 * H) - 2 * oh) * 2 + (am % (2 * H) - 2 * ow)
        code = v[key].reshape(Bn, H, H, C).transpose(0, 3, 1, 2).astype(np.int64) & 3
        agree = float((code == pos).mean())
        print(f"B={Bn} {key} argmax agreement {agree:.5f}")
        assert agree > ARGMAX_AGREE[key], (key, agree)


def test_loss_grads_update(large_step):
    s = large_step
    w, ref, Bn = s["w"], s["ref"], s["B"]
    lerr = abs(s["gl"] - s["rl"]) / abs(s["rl"])
    errs = {name: npref.normwise(s["grads"][o:o + n], ref.grads[o:o + n]) for name, o, n in blocks(w)}
    perr = npref.normwise(s["params"], ref.params)
    print(f"B={Bn} loss relative error {lerr:.2e}; weights after Adam {perr:.2e}")
    print(f"B={Bn} gradient normwise errors:", {k: f"{e:.2e}" for k, e in errs.items()})
    assert lerr < LOSS_TOL, (s["gl"], s["rl"])
    assert all(e < GRAD_TOL[Bn] for e in errs.values()), errs
    assert perr < 1e-2


def test_adam_trajectory_follows_fp32_engine():
    """Five Adam steps of the large CNN at the 8-GPU per-rank batch (1024) on both engines
    from the same weights and batches: the bf16 engine's losses stay within TRAJ_TOL
    (relative) of the fp32 engine's, which matches the oracle to 1e-5."""
    w, Bn = configs.CNN_LARGE, 1024
    p0 = synthetic.init_params(w, seed=17)
    nets = [Net(w, batch=Bn, precision=p) for p in (0, 1)]
    for n in nets:
        n.set_params(p0)
    worst = 0.0
    for k in range(5):
        x, y = synthetic.batch(w, Bn, seed=17, step=k)
        l32, l16 = (n.step_host(x, y) for n in nets)
        worst = max(worst, abs(l16 - l32) / abs(l32))
        print(f"step {k}: fp32 engine {l32 / Bn:.6f}  bf16 engine {l16 / Bn:.6f}")
    pe = npref.normwise(nets[1].params(), nets[0].params())
    print(f"trajectory: worst loss relative gap {worst:.2e}, weights after 5 steps {pe:.2e}")
    for n in nets:
        n.close()
    assert worst < TRAJ_TOL
    assert pe < 1e-2


def test_deterministic():
    w = configs.CNN_LARGE
    p0 = synthetic.init_params(w, seed=4)
    x, y = synthetic.batch(w, 128, seed=4)
    a, b = Net(w, batch=128, precision=1), Net(w, batch=128, precision=1)
    a.set_params(p0); b.set_params(p0)
    la, lb = a.step_host(x, y, update=False), b.step_host(x, y, update=False)
    assert la == lb
    assert np.array_equal(a.grads(), b.grads())
    a.close(); b.close()
