"""The bf16 tcgen05 engine on the audio keyword CNN (GPU): Conv(1->16) + ReLU +
Pool -> Conv(16->32) + ReLU + Pool -> Conv(32->64) + ReLU + Pool ->
Linear(6144->12) on 1x64x101 log-mel inputs (odd widths: floor pooling drops
the last column of the 101- and 25-wide maps).

Kernel level (batches 64 and 4096, the benchmarked batch): every contraction
is recomputed in float64 from the engine's own inputs (its bf16 intermediates,
read through zilla_net_inspect; PyTorch on the GPU as the checker):
  bf16 outputs (activations, activation gradients)   normwise <= 1e-2
  fp32 outputs (logit, weight and bias gradients)    normwise <= 2e-3
  unpool routing (argmax + ReLU codes, zero columns) exact
End to end against the fp32 oracle (batch 64 and 512), measured values in
brackets: activations within 2e-2 [2.7e-3 .. 6.2e-3], pool argmax agreement
above 99% [99.3% .. 100%], loss within 5e-3 relative [2.1e-3, 2.4e-3],
gradient blocks within 0.1 normwise [1.5e-3 .. 2.0e-2], weights after one
Adam step within 1e-2 [2.5e-3].  The loss bar is wider than the large CNN's
(1e-3): the untrained net's logits on these N(-4, 2^2) spectrograms reach
about 30, so the 2^-9 relative rounding of the bf16 activations shows up in
the loss at about that size.
"""
import os

import numpy as np
import pytest

import npref
import oracle
from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import Net
from test_tc_kernels_gpu import T, bf16, conv_dgrad, conv_fwd, conv_wgrad, normwise, unpool

pytestmark = pytest.mark.gpu
W = configs.AUDIO_CNN


def pool_floor(c):
    """2x2/2 max-pool of NHWC with floor: a trailing odd row / column is dropped."""
    import torch
    Ho, Wo = c.shape[1] // 2, c.shape[2] // 2
    return torch.stack([c[:, dh:2 * Ho:2, dw:2 * Wo:2, :] for dh in (0, 1) for dw in (0, 1)], -1).amax(-1)


def param_views(w, flat):
    P, off = {}, 0
    for li, (kind, a, b, _) in enumerate(w.layers):
        if kind == configs.CONV:
            P[f"W{li}"] = (off, (b, a, 3, 3)); off += b * a * 9
            P[f"b{li}"] = (off, (b,)); off += b
        elif kind == configs.LINEAR:
            P[f"W{li}"] = (off, (a, b)); off += a * b
            P[f"b{li}"] = (off, (b,)); off += b
    return {k: flat[o:o + int(np.prod(s))].reshape(s) for k, (o, s) in P.items()}


@pytest.fixture(scope="module", params=(64, 4096), ids=("B64", "B4096"))
def step(request):
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    B = request.param
    p0 = synthetic.init_params(W, seed=41)
    x, y = synthetic.batch(W, B, seed=41)
    net = Net(W, batch=B, precision=1)
    net.set_params(p0)
    net.step_host(x, y, update=False)
    net.device_status()
    v = {k: T(a) for k, a in net.inspect().items()}
    g = net.grads()
    net.close()
    yield dict(B=B, x=T(x.reshape(B, 64, 101, 1)), y=torch.from_numpy(y.astype(np.int64)).cuda(), v=v,
               par=param_views(W, p0), grd={k: T(a) for k, a in param_views(W, g).items()})
    torch.cuda.empty_cache()


def check(step, name, got, ref, tol):
    e = normwise(got, ref)
    print(f"audio B={step['B']} {name}: normwise {e:.2e}")
    assert e < tol, (step["B"], name, e)


def test_forward_kernels(step):
    B, v, par = step["B"], step["v"], step["par"]
    c1 = (conv_fwd(step["x"], T(par["W0"])) + T(par["b0"])).clamp_min(0)
    check(step, "conv1 fwd+pool (bf16)", v["conv1.out"].reshape(B, 32, 50, 16), pool_floor(c1), 1e-2)
    del c1
    a1 = v["conv1.out"].reshape(B, 32, 50, 16)
    c2 = (conv_fwd(a1, T(bf16(par["W3"]))) + T(par["b3"])).clamp_min(0)
    check(step, "conv2 fwd+pool (bf16)", v["conv2.out"].reshape(B, 16, 25, 32), pool_floor(c2), 1e-2)
    del c2
    p2 = v["conv2.out"].reshape(B, 16, 25, 32)
    c3 = (conv_fwd(p2, T(bf16(par["W6"]))) + T(par["b6"])).clamp_min(0)
    check(step, "conv3 fwd+pool (bf16)", v["conv3.out"].reshape(B, 8, 12, 64), pool_floor(c3), 1e-2)


def test_head(step):
    import torch
    B, v, par, grd = step["B"], step["v"], step["par"], step["grd"]
    flat = v["conv3.out"].reshape(B, 6144)                                 # NHWC flatten
    perm = np.arange(6144).reshape(64, 8, 12).transpose(1, 2, 0).ravel()   # NHWC pos -> NCHW row
    W9 = T(bf16(par["W9"]))[perm]                                          # bf16 weights, NHWC rows
    z = flat @ W9 + T(par["b9"])
    dz = torch.softmax(z, 1)
    dz[torch.arange(B, device="cuda"), step["y"]] -= 1
    dz /= B
    check(step, "head dz (fp32)", v["head.dz"].reshape(B, 12), dz, 2e-3)
    dzg = v["head.dz"].reshape(B, 12)
    check(step, "head dX (bf16)", v["flat.d"].reshape(B, 6144), dzg @ W9.T, 1e-2)
    dW = T(np.zeros((6144, 12)))
    dW[perm] = flat.T @ dzg
    check(step, "head dW", grd["W9"], dW, 2e-3)
    check(step, "head db", grd["b9"], dzg.sum(0), 2e-3)


def test_conv_backward(step):
    B, v, par, grd = step["B"], step["v"], step["par"], step["grd"]
    code3 = v["conv3.code"].reshape(B, 8, 12, 64).long()
    dC3 = unpool(v["flat.d"].reshape(B, 8, 12, 64), code3, 16, 25)
    assert bool((v["conv3.dC"].reshape(B, 16, 25, 64) == dC3).all()), "unpool3 routing"
    check(step, "db conv3", grd["b6"], dC3.sum((0, 1, 2)), 2e-3)
    p2 = v["conv2.out"].reshape(B, 16, 25, 32)
    check(step, "conv3 dW", grd["W6"], conv_wgrad(p2, dC3), 2e-3)
    check(step, "conv3 dX (bf16)", v["conv2.dP"].reshape(B, 16, 25, 32), conv_dgrad(dC3, T(bf16(par["W6"]))), 1e-2)
    del dC3
    code2 = v["conv2.code"].reshape(B, 16, 25, 32).long()
    dC2 = unpool(v["conv2.dP"].reshape(B, 16, 25, 32), code2, 32, 50)
    assert bool((v["conv2.dC"].reshape(B, 32, 50, 32) == dC2).all()), "unpool2 routing"
    check(step, "db conv2", grd["b3"], dC2.sum((0, 1, 2)), 2e-3)
    a1 = v["conv1.out"].reshape(B, 32, 50, 16)
    check(step, "conv2 dW", grd["W3"], conv_wgrad(a1, dC2), 2e-3)
    check(step, "conv2 dX (bf16)", v["conv1.dP"].reshape(B, 32, 50, 16), conv_dgrad(dC2, T(bf16(par["W3"]))), 1e-2)
    del dC2
    code1 = v["conv1.code"].reshape(B, 32, 50, 16).long()
    dC1 = unpool(v["conv1.dP"].reshape(B, 32, 50, 16), code1, 64, 101)
    if "conv1.dC" in v:   # else the weight-gradient kernel builds dC1 itself from dP1 and the codes
        assert bool((v["conv1.dC"].reshape(B, 64, 101, 16) == dC1).all()), "unpool1 routing"
    check(step, "conv1 dW", grd["W0"], conv_wgrad(step["x"], dC1), 2e-3)
    check(step, "db conv1", grd["b0"], dC1.sum((0, 1, 2)), 2e-3)


@pytest.mark.parametrize("B", (64, 512))
def test_against_oracle(B):
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else 1
    p0 = synthetic.init_params(W, seed=43)
    x, y = synthetic.batch(W, B, seed=43)
    ref = oracle.StepModel(W.spec(), B, W.in_shape, nthreads=threads)
    ref.params[:] = p0
    rl = ref.step(x, y, W.optimizer, W.lr)
    net = Net(W, batch=B, precision=1)
    try:
        net.set_params(p0)
        gl = net.step_host(x, y)
        net.device_status()
        v = net.inspect()
        g, pa = net.grads(), net.params()
    finally:
        net.close()

    def nhwc(a, C, H, Wd):
        return a.reshape(B, C, H, Wd).transpose(0, 2, 3, 1).ravel()

    # oracle layer outputs (NCHW fp32): 2 pool1, 5 pool2, 8 pool3
    errs = {"conv1": npref.normwise(v["conv1.out"], nhwc(ref.output(2, B * 16 * 32 * 50), 16, 32, 50)),
            "conv2": npref.normwise(v["conv2.out"], nhwc(ref.output(5, B * 32 * 16 * 25), 32, 16, 25)),
            "conv3": npref.normwise(v["conv3.out"], nhwc(ref.output(8, B * 64 * 8 * 12), 64, 8, 12))}
    print(f"audio B={B} forward normwise errors:", errs)
    assert all(e < 2e-2 for e in errs.values()), errs
    for layer, C, Ho, Wo, Wi, key in ((2, 16, 32, 50, 101, "conv1.code"), (5, 32, 16, 25, 50, "conv2.code"),
                                      (8, 64, 8, 12, 25, "conv3.code")):
        am = ref.argmax(layer, B * C * Ho * Wo).reshape(B, C, Ho, Wo)
        oh = np.arange(Ho)[:, None]; ow = np.arange(Wo)[None, :]
        pos = (am // Wi - 2 * oh) * 2 + (am % Wi - 2 * ow)
        code = v[key].reshape(B, Ho, Wo, C).transpose(0, 3, 1, 2).astype(np.int64) & 3
        agree = float((code == pos).mean())
        print(f"audio B={B} {key} argmax agreement {agree:.5f}")
        assert agree > 0.99, (key, agree)
    lerr = abs(gl - rl) / abs(rl)
    blocks = {k: npref.normwise(a, b) for (k, a), b in zip(param_views(W, g).items(), param_views(W, ref.grads).values())}
    perr = npref.normwise(pa, ref.params)
    print(f"audio B={B} loss relative error {lerr:.2e}; weights after Adam {perr:.2e}")
    print(f"audio B={B} gradient normwise errors:", {k: f"{e:.2e}" for k, e in blocks.items()})
    assert lerr < 5e-3, (gl, rl)
    assert all(e < 0.1 for e in blocks.values()), blocks
    assert perr < 1e-2
