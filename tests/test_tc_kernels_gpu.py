"""Kernel-level parity of the bf16 tcgen05 engine (GPU), at the per-GPU batches
the step is benchmarked at.

Every contraction of the large-CNN step is recomputed in float64 from the
engine's own inputs (its bf16 intermediates, read through zilla_net_inspect),
so the only remaining difference is fp32 accumulation / bf16 output rounding:
  bf16 outputs (activations, activation gradients)   normwise <= 1e-2
  fp32 outputs (weight / bias gradients)             normwise <= 2e-3
  unpool routing (argmax + ReLU codes)               exact
The float64 references run in PyTorch on the same GPU (checker only: cuDNN /
cuBLAS in float64, no TF32).  Batches: 16 (a partial first wave), 1024 (the
per-rank batch of 8 GPUs: fewer tiles than CTA slots, one-wave split-K
choices) and 8192 (one GPU: many waves, the widest splits).  End-to-end
differences against the fp32 oracle come on top of this from ReLU-mask and
max-pool decisions that bf16 rounding flips near ties; those are checked in
test_tc_gpu.py.
"""
import numpy as np
import pytest

from zillaphp_b200 import configs, synthetic
from zillaphp_b200.net import Net

pytestmark = pytest.mark.gpu
BATCHES = (16, 1024, 8192)


def T(a):
    """float64 CUDA tensor of a host array."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda", torch.float64)


def bf16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).float().numpy()


def nchw(x):
    return x.permute(0, 3, 1, 2).contiguous()


def nhwc(x):
    return x.permute(0, 2, 3, 1).contiguous()


def conv_fwd(x, Wt):           # x NHWC, Wt [co][ci][3][3]: 3x3, pad 1
    import torch.nn.functional as F
    return nhwc(F.conv2d(nchw(x), Wt, padding=1))


def conv_dgrad(dy, Wt):        # dx[b,i,j,ci] = sum dy[b, i-dh+1, j-dw+1, co] W[co,ci,dh,dw]
    import torch.nn.functional as F
    return nhwc(F.conv_transpose2d(nchw(dy), Wt, padding=1))


def conv_wgrad(x, dy):         # dW[co,ci,dh,dw] = sum x[b, h+dh-1, w+dw-1, ci] dy[b,h,w,co]
    import torch
    return torch.nn.grad.conv2d_weight(nchw(x), (dy.shape[3], x.shape[3], 3, 3), nchw(dy), padding=1)


def pool(c):                   # 2x2 max-pool of NHWC
    import torch
    return torch.stack([c[:, dh::2, dw::2, :] for dh in (0, 1) for dw in (0, 1)], -1).amax(-1)


def unpool(dp, code, H, W):
    import torch
    Bn, Ho, Wo, C = dp.shape
    out = torch.zeros((Bn, H, W, C), dtype=dp.dtype, device=dp.device)
    for ph in (0, 1):
        for pw in (0, 1):
            hit = ((code & 3) == (ph * 2 + pw)) & ((code & 4) != 0)
            out[:, ph:2 * Ho:2, pw:2 * Wo:2, :] = torch.where(hit, dp, torch.zeros_like(dp))
    return out


def normwise(got, ref):
    import torch
    got, ref = got.to(torch.float64), ref.to(torch.float64)
    return float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


@pytest.fixture(scope="module", params=BATCHES, ids=[f"B{b}" for b in BATCHES])
def step(request):
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    B = request.param
    w = configs.CNN_LARGE
    p0 = synthetic.init_params(w, seed=33)
    x, y = synthetic.batch(w, B, seed=33)
    net = Net(w, batch=B, precision=1)
    net.set_params(p0)
    net.step_host(x, y, update=False)
    net.device_status()
    v = {k: T(a) for k, a in net.inspect().items()}
    g = net.grads()
    net.close()
    P, off = {}, 0   # parameter views (Sequential order)
    for li, (kind, a, b, _) in enumerate(w.layers):
        if kind == configs.CONV:
            P[f"W{li}"] = (off, (b, a, 3, 3)); off += b * a * 9
            P[f"b{li}"] = (off, (b,)); off += b
        elif kind == configs.LINEAR:
            P[f"W{li}"] = (off, (a, b)); off += a * b
            P[f"b{li}"] = (off, (b,)); off += b
    par = {k: p0[o:o + int(np.prod(s))].reshape(s) for k, (o, s) in P.items()}
    grd = {k: T(g[o:o + int(np.prod(s))].reshape(s)) for k, (o, s) in P.items()}
    yield dict(B=B, x=T(x.reshape(B, 28, 28, 1)), y=torch.from_numpy(y.astype(np.int64)).cuda(), v=v,
               par=par, grd=grd)
    torch.cuda.empty_cache()


def check(step, name, got, ref, tol):
    e = normwise(got, ref)
    print(f"B={step['B']} {name}: normwise {e:.2e}")
    assert e < tol, (step["B"], name, e)


def test_head(step):
    import torch
    B, v, par, grd = step["B"], step["v"], step["par"], step["grd"]
    a4 = v["hidden.out"].reshape(B, 256)
    W10 = T(par["W10"])
    z = a4 @ W10 + T(par["b10"])
    p = torch.softmax(z, 1)
    dz = p.clone()
    dz[torch.arange(B, device="cuda"), step["y"]] -= 1
    dz /= B
    da = (dz @ W10.T) * (a4 > 0)
    check(step, "head dA (bf16)", v["hidden.dZ"].reshape(B, 256), da, 1e-2)
    check(step, "dW fc2", grd["W10"], a4.T @ dz, 2e-3)
    check(step, "db fc2", grd["b10"], dz.sum(0), 2e-3)
    check(step, "db fc1", grd["b8"], da.sum(0), 2e-3)


def test_fc1_backward(step):
    B, v, par, grd = step["B"], step["v"], step["par"], step["grd"]
    dz4 = v["hidden.dZ"].reshape(B, 256)
    p3 = v["conv3.out"].reshape(B, 7 * 7 * 128)                            # NHWC flatten
    perm = np.arange(6272).reshape(128, 7, 7).transpose(1, 2, 0).ravel()   # NHWC pos -> NCHW row
    W4 = T(bf16(par["W8"]))                                                # [6272 (NCHW), 256]
    check(step, "fc1 dX (bf16)", v["flat.d"].reshape(B, 6272), dz4 @ W4[perm].T, 1e-2)
    dW = T(np.zeros((6272, 256)))
    dW[perm] = p3.T @ dz4
    check(step, "fc1 dW", grd["W8"], dW, 2e-3)


def test_conv_backward(step):
    B, v, par, grd = step["B"], step["v"], step["par"], step["grd"]
    p2 = v["conv2.out"].reshape(B, 14, 14, 64)
    a1 = v["conv1.out"].reshape(B, 28, 28, 32)
    code3 = v["conv3.code"].reshape(B, 7, 7, 128).long()
    code2 = v["conv2.code"].reshape(B, 14, 14, 64).long()
    dC3 = unpool(v["flat.d"].reshape(B, 7, 7, 128), code3, 14, 14)
    if "conv3.dC" in v:   # else conv3's backward kernels build dC3 on chip from dP3 and the codes
        assert bool((v["conv3.dC"].reshape(B, 14, 14, 128) == dC3).all()), "unpool3 routing"
    check(step, "db conv3", grd["b5"], dC3.sum((0, 1, 2)), 2e-3)
    check(step, "conv3 dX (bf16)", v["conv2.dP"].reshape(B, 14, 14, 64), conv_dgrad(dC3, T(bf16(par["W5"]))), 1e-2)
    check(step, "conv3 dW", grd["W5"], conv_wgrad(p2, dC3), 2e-3)
    dC2 = unpool(v["conv2.dP"].reshape(B, 14, 14, 64), code2, 28, 28)
    if "conv2.dC" in v:   # else dC2 is built on chip by conv2's backward kernel from dP2 and the codes
        assert bool((v["conv2.dC"].reshape(B, 28, 28, 64) == dC2).all()), "unpool2 routing"
    check(step, "db conv2", grd["b2"], dC2.sum((0, 1, 2)), 2e-3)
    dC1_ref = conv_dgrad(dC2, T(bf16(par["W2"]))) * (a1 > 0)
    if "conv1.dC" in v:   # input gradient of conv2 written to global memory
        check(step, "conv2 dX*mask (bf16)", v["conv1.dC"].reshape(B, 28, 28, 32), dC1_ref, 1e-2)
        dC1 = v["conv1.dC"].reshape(B, 28, 28, 32)
    else:                 # kept on chip: conv1's weight gradient is taken in conv2's backward kernel
        dC1 = T(bf16(dC1_ref.cpu().numpy()))
    del dC1_ref
    check(step, "conv2 dW", grd["W2"], conv_wgrad(a1, dC2), 2e-3)
    del dC2
    check(step, "conv1 dW", grd["W0"], conv_wgrad(step["x"], dC1), 2e-3)
    check(step, "db conv1", grd["b0"], dC1.sum((0, 1, 2)), 2e-3)


def test_forward_kernels(step):
    B, v, par = step["B"], step["v"], step["par"]
    a1 = (conv_fwd(step["x"], T(par["W0"])) + T(par["b0"])).clamp_min(0)
    check(step, "conv1 fwd (bf16)", v["conv1.out"].reshape(B, 28, 28, 32), a1, 1e-2)
    del a1
    a1b = v["conv1.out"].reshape(B, 28, 28, 32)
    c2 = (conv_fwd(a1b, T(bf16(par["W2"]))) + T(par["b2"])).clamp_min(0)
    check(step, "conv2 fwd+pool (bf16)", v["conv2.out"].reshape(B, 14, 14, 64), pool(c2), 1e-2)
    del c2
    p2 = v["conv2.out"].reshape(B, 14, 14, 64)
    c3 = (conv_fwd(p2, T(bf16(par["W5"]))) + T(par["b5"])).clamp_min(0)
    check(step, "conv3 fwd+pool (bf16)", v["conv3.out"].reshape(B, 7, 7, 128), pool(c3), 1e-2)
    p3 = v["conv3.out"].reshape(B, 6272)
    perm = np.arange(6272).reshape(128, 7, 7).transpose(1, 2, 0).ravel()
    a4 = (p3 @ T(bf16(par["W8"]))[perm] + T(par["b8"])).clamp_min(0)
    check(step, "fc1 fwd (bf16)", v["hidden.out"].reshape(B, 256), a4, 1e-2)


def test_pool_codes_follow_the_rounded_conv(step):
    """The pool codes name the window position of the first maximum of conv2's outputs
    (after bias and ReLU, rounded to bf16) and flag a positive maximum.  Recomputed in
    float64 from the engine's own inputs, the positions agree except where the window's
    two largest values lie within bf16 rounding (2^-7 relative) of each other, and the
    flags agree except where the pre-ReLU maximum is within 1e-3 of the layer's largest
    magnitude of zero: near-ties that fp32 accumulation order decides."""
    import torch
    B, v, par = step["B"], step["v"], step["par"]
    a1b = v["conv1.out"].reshape(B, 28, 28, 32)
    pre = conv_fwd(a1b, T(bf16(par["W2"]))) + T(par["b2"])
    win = torch.stack([pre[:, dh::2, dw::2, :] for dh in (0, 1) for dw in (0, 1)], -1)   # [B,14,14,64,4]
    del pre
    best = win.amax(-1)
    relu = win.clamp_min(0)
    pos = (relu == relu.amax(-1, keepdim=True)).to(torch.int8).argmax(-1)   # first maximum, (kh, kw) order
    srt = relu.sort(-1, descending=True).values
    near = (srt[..., 0] - srt[..., 1]) <= srt[..., 0] * 2.0 ** -7
    code = v["conv2.code"].reshape(B, 14, 14, 64).long()
    agree = (code & 3) == pos
    print(f"B={B} pool2 position agreement with the float64 recomputation: {float(agree.double().mean()):.6f}")
    assert bool((agree | near).all()), "a pool position disagrees away from a near-tie"
    flag = ((code >> 2) & 1) == (best > 0).long()
    zero_tie = best.abs() <= 1e-3 * float(win.abs().max())
    print(f"B={B} pool2 ReLU-flag agreement: {float(flag.double().mean()):.6f}")
    assert bool((flag | zero_tie).all()), "a ReLU flag disagrees away from zero"
