"""Every reference entry point on the B200 against the CPU oracle (GPU).

Calls go through the C-ABI (B200Backend mirrors CudaBackend.php).  Bars:
bit-exact for argmax / integer work and for the forward contractions that
follow the reference's summation order (conv forward, matmul_dev); 1e-4
normwise for the other float reductions (different summation order).
"""
import numpy as np
import pytest

import npref
import oracle
from zillaphp_b200.backend import B200Backend, ZillaError

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    return B200Backend()


def put(be, a):
    a = np.ascontiguousarray(a, np.float32).ravel()
    i = be.bufferAlloc(max(a.size, 1))
    if a.size:
        be.bufferUpload(i, a)
    return i


def get(be, i, n, shape=None):
    out = be.bufferDownload(i, n)
    return out.reshape(shape) if shape else out


def test_reference_known_answers(be, golden):
    g = golden["conv2d_1x4x4"]
    ids = [put(be, g["input"]), put(be, g["weight"]), put(be, g["bias"]), be.bufferAlloc(4)]
    be.conv2dFwdDev(*ids, 1, 4, 4, 1, 2, 2, 3, 3, 1, 0)
    np.testing.assert_allclose(get(be, ids[3], 4), g["expected"], atol=g["tol"])
    g = golden["conv2d_batched"]
    ids = [put(be, g["input"]), put(be, g["weight"]), put(be, g["bias"]), be.bufferAlloc(8)]
    be.conv2dBatchedFwdDev(*ids, 2, 1, 4, 4, 1, 2, 2, 3, 3, 1, 0)
    np.testing.assert_allclose(get(be, ids[3], 8), g["expected"], atol=g["tol"])
    g = golden["matmul_2x2"]
    a, b, c = put(be, g["a"]), put(be, g["b"]), be.bufferAlloc(4)
    be.matmulDev(a, b, c, 2, 2, 2)
    assert get(be, c, 4).tolist() == g["expected"]
    assert be.matmul(np.array(g["a"]).reshape(2, 2), np.array(g["b"]).reshape(2, 2)).ravel().tolist() == g["expected"]
    g = golden["softmax_rows"]
    x, y = put(be, g["x"]), be.bufferAlloc(20)
    be.softmaxRowsFwdDev(x, y, 4, 5)
    np.testing.assert_allclose(get(be, y, 20), g["expected"], atol=g["tol"])
    g = golden["causal_softmax"]
    x = put(be, g["x"])
    be.causalSoftmaxDev(x, 4, 4, g["mask"])
    np.testing.assert_allclose(get(be, x, 16), g["expected"], atol=g["tol"])
    g = golden["scale"]
    x = put(be, g["x"])
    be.scaleDev(x, g["s"], 6)
    np.testing.assert_allclose(get(be, x, 6), g["expected"], atol=g["tol"])
    g = golden["softmax_bwd"]
    p, dp, ds = put(be, g["P"]), put(be, g["dP"]), be.bufferAlloc(6)
    be.softmaxRowsBwdDev(p, dp, ds, 2, 3)
    np.testing.assert_allclose(get(be, ds, 6), g["expected"], atol=g["tol"])
    g = golden["relu"]
    x, y = put(be, g["x"]), be.bufferAlloc(4)
    be.reluDev(x, y, 4)
    assert get(be, y, 4).tolist() == g["expected"]


@pytest.mark.parametrize("B,C,H,W,oC,pad,stride", [(2, 1, 28, 28, 8, 0, 1), (3, 5, 13, 11, 7, 1, 1),
                                                   (2, 3, 9, 9, 4, 1, 2), (1, 16, 32, 50, 32, 1, 1),
                                                   (4, 32, 14, 14, 64, 1, 1)])
def test_conv_batched_matches_oracle(be, B, C, H, W, oC, pad, stride):
    g = np.random.default_rng(B * 100 + C)
    x = g.standard_normal((B, C, H, W)).astype(np.float32)
    w = (g.standard_normal((oC, C, 3, 3)) * 0.3).astype(np.float32)
    b = g.standard_normal(oC).astype(np.float32)
    oH, oW = (H + 2 * pad - 3) // stride + 1, (W + 2 * pad - 3) // stride + 1
    ref = oracle.conv2d_batched_forward(x, w, b, stride, pad)
    ix, iw, ib, iy = put(be, x), put(be, w), put(be, b), be.bufferAlloc(B * oC * oH * oW)
    be.conv2dBatchedFwdDev(ix, iw, ib, iy, B, C, H, W, oC, oH, oW, 3, 3, stride, pad)
    got = get(be, iy, B * oC * oH * oW, ref.shape)
    assert np.array_equal(got, ref), npref.normwise(got, ref)   # reference summation order
    go = g.standard_normal(ref.shape).astype(np.float32)
    rgx, rgw, rgb = oracle.conv2d_batched_backward(x, w, go, stride, pad)
    igo, igx, igw, igb = put(be, go), be.bufferAlloc(x.size), be.bufferAlloc(w.size), be.bufferAlloc(oC)
    be.conv2dBatchedBwdDev(ix, iw, igo, igx, igw, igb, B, C, H, W, oC, oH, oW, 3, 3, stride, pad)
    assert npref.normwise(get(be, igx, x.size, x.shape), rgx) < 1e-5
    assert npref.normwise(get(be, igw, w.size, w.shape), rgw) < 1e-5
    assert npref.normwise(get(be, igb, oC), rgb) < 1e-5
    if B == 1:
        iy1 = be.bufferAlloc(oC * oH * oW)
        be.conv2dFwdDev(ix, iw, ib, iy1, C, H, W, oC, oH, oW, 3, 3, stride, pad)
        assert np.array_equal(get(be, iy1, oC * oH * oW, ref.shape), ref)


@pytest.mark.parametrize("B,C,H,W", [(2, 3, 28, 28), (3, 4, 64, 101), (1, 2, 5, 7), (2, 8, 25, 25)])
def test_maxpool_matches_oracle_bit_exact(be, B, C, H, W):
    g = np.random.default_rng(H * W)
    x = np.maximum(g.standard_normal((B, C, H, W)), 0).astype(np.float32)   # zero ties
    x[0, 0, :2, :2] = 0.0
    ref_out, ref_arg = oracle.maxpool2d_batched_forward(x)
    oH, oW = ref_out.shape[2:]
    n = B * C * oH * oW
    ix, io, ia = put(be, x), be.bufferAlloc(n), be.bufferAlloc(n)
    be.maxPool2dBatchedFwdDev(ix, io, ia, B, C, H, W, oH, oW, 2, 2, 2)
    assert np.array_equal(get(be, io, n, ref_out.shape), ref_out)
    assert np.array_equal(be.bufferDownloadInt(ia, n).reshape(ref_arg.shape), ref_arg)
    go = g.standard_normal(ref_out.shape).astype(np.float32)
    igo, igi = put(be, go), be.bufferAlloc(x.size)
    be.zeroDev(igi, x.size)                                    # caller zeroes, as the reference
    be.maxPool2dBatchedBwdDev(igo, ia, igi, B, C, oH, oW)
    ref_gi = np.stack([oracle.maxpool2d_backward(go[i], oracle.maxpool2d_forward(x[i])[1], H, W) for i in range(B)])
    assert np.array_equal(get(be, igi, x.size, x.shape), ref_gi)
    # per-sample entry points: channel-inclusive, sample-local argmax
    ix1, io1, ia1 = put(be, x[0]), be.bufferAlloc(n // B), be.bufferAlloc(n // B)
    be.maxPool2dFwdDev(ix1, io1, ia1, C, H, W, oH, oW, 2, 2, 2)
    assert np.array_equal(be.bufferDownloadInt(ia1, n // B), ref_arg[0].ravel())


def test_maxpool_backward_rejects_out_of_range_argmax(be):
    igo, ia, igi = put(be, np.ones(4)), be.bufferAlloc(4), be.bufferAlloc(8)
    be.bufferUploadInt(ia, np.array([0, 3, 7, 1000000], np.int32))
    be.zeroDev(igi, 8)
    be.maxPool2dBatchedBwdDev(igo, ia, igi, 1, 1, 2, 2)
    got = get(be, igi, 8)
    assert got.tolist() == [1, 0, 0, 1, 0, 0, 0, 1]          # index 1000000 skipped
    assert be.ffi.zilla_check_device() == -3                 # ... and reported
    assert be.ffi.zilla_check_device() == 0                  # read-and-clear


@pytest.mark.parametrize("M,K,N", [(64, 784, 128), (64, 128, 10), (7, 33, 5), (300, 257, 65), (1, 1, 1)])
def test_matmul_variants(be, M, K, N):
    g = np.random.default_rng(M + K + N)
    a = g.standard_normal((M, K)).astype(np.float32)
    b = g.standard_normal((K, N)).astype(np.float32)
    ia, ib, ic = put(be, a), put(be, b), be.bufferAlloc(M * N)
    be.matmulDev(ia, ib, ic, M, K, N)
    assert np.array_equal(get(be, ic, M * N, (M, N)), oracle.matmul_dev(a, b, "nn"))
    at, bt = put(be, a.T.copy()), put(be, b.T.copy())
    be.matmulTnDev(at, ib, ic, M, K, N)
    assert npref.normwise(get(be, ic, M * N, (M, N)), oracle.matmul_dev(a.T.copy(), b, "tn")) < 1e-5
    be.matmulNtDev(ia, bt, ic, M, K, N)
    assert npref.normwise(get(be, ic, M * N, (M, N)), oracle.matmul_dev(a, b.T.copy(), "nt")) < 1e-5
    assert npref.normwise(be.matmul(a, b), oracle.matmul(a, b)) < 1e-5


@pytest.mark.parametrize("B,C", [(64, 10), (8192, 10), (37, 65), (3, 129), (5, 1)])
def test_softmax_ce_bias_grad(be, B, C):
    g = np.random.default_rng(B * C)
    z = (g.standard_normal((B, C)) * 4).astype(np.float32)
    t = g.integers(0, C, B).astype(np.float32)
    iz, it, idz, il = put(be, z), put(be, t), be.bufferAlloc(B * C), put(be, [0.0])
    be.softmaxCeDev(iz, it, idz, il, B, C)
    dz = get(be, idz, B * C, (B, C))
    loss = get(be, il, 1)[0]
    if C <= 128:
        rdz, rl = oracle.softmax_ce_dev(z, t)
    else:   # the CPU reference rejects C > 128; compare with the float64 statement
        e = np.exp(z - z.max(1, keepdims=True)); p = e / e.sum(1, keepdims=True)
        rl = -np.log(p[np.arange(B), t.astype(int)]).sum(); rdz = p.copy(); rdz[np.arange(B), t.astype(int)] -= 1; rdz /= B
    assert npref.normwise(dz, rdz) < 1e-5
    assert abs(loss - rl) / max(abs(rl), 1e-6) < 1e-5
    be.softmaxCeDev(iz, it, idz, il, B, C)                   # accumulates into *loss
    assert abs(get(be, il, 1)[0] - 2 * rl) / max(abs(rl), 1e-6) < 1e-5
    idb = be.bufferAlloc(C)
    be.biasGradDev(idz, idb, B, C)
    assert npref.normwise(get(be, idb, C), oracle.bias_grad_dev(dz)) < 1e-5


def test_elementwise_relu_sgd_adam_copy(be):
    g = np.random.default_rng(5)
    n = 100_003
    a = g.standard_normal(n).astype(np.float32)
    b = (g.standard_normal(n) + 3).astype(np.float32)
    ia, ib, ic = put(be, a), put(be, b), be.bufferAlloc(n)
    for op, ref in (("addDev", a + b), ("subDev", a - b), ("mulDev", a * b), ("divDev", a / b)):
        getattr(be, op)(ia, ib, ic, n)
        assert np.array_equal(get(be, ic, n), ref), op
    for op, ref in (("add", a + b), ("sub", a - b), ("mul", a * b), ("div", a / b)):
        assert np.array_equal(be.elementwise(op, a, b), ref)
    assert np.array_equal(be.elementwise("relu", a), np.maximum(a, 0))
    iy, im = be.bufferAlloc(n), be.bufferAlloc(n)
    be.reluFwdDev(ia, iy, im, n)
    ry, rm = oracle.relu_fwd_dev(a)
    assert np.array_equal(get(be, iy, n), ry) and np.array_equal(get(be, im, n), rm)
    be.reluBwdDev(ib, im, ic, n)
    assert np.array_equal(get(be, ic, n), oracle.relu_bwd_dev(b, rm))
    be.sgdUpdateDev(ia, ib, 0.05, n)
    assert np.array_equal(get(be, ia, n), oracle.sgd_update_dev(a, b, 0.05))
    be.copyDev(ib, ic, n)
    assert np.array_equal(get(be, ic, n), b)
    be.zeroDev(ic, n)
    assert not get(be, ic, n).any()
    x = np.arange(12, dtype=np.float32).reshape(3, 4)
    ix = put(be, x)
    be.addBiasDev(ix, put(be, [1, 2, 3, 4]), 3, 4)
    assert np.array_equal(get(be, ix, 12, (3, 4)), oracle.add_bias_dev(x, [1, 2, 3, 4]))
    # Adam against the restated PHP optimizer, three steps
    w0 = g.standard_normal(n).astype(np.float32)
    iw, ig, im_, iv = put(be, w0), be.bufferAlloc(n), be.bufferAlloc(n), be.bufferAlloc(n)
    be.zeroDev(im_, n); be.zeroDev(iv, n)
    rw, rm_, rv = w0, np.zeros(n, np.float32), np.zeros(n, np.float32)
    for t in (1, 2, 3):
        gr = g.standard_normal(n).astype(np.float32)
        be.bufferUpload(ig, gr)
        be.adamUpdateDev(iw, ig, im_, iv, 1e-3, 0.9, 0.999, 1e-8, t, n)
        rw, rm_, rv = oracle.adam_update(rw, gr, rm_, rv, 1e-3, t=t)
    assert npref.normwise(get(be, iw, n), rw) < 1e-6


def test_attention_primitives(be):
    g = np.random.default_rng(9)
    N, M = 33, 300
    x = (g.standard_normal((N, M)) * 3).astype(np.float32)
    ix, iy = put(be, x), be.bufferAlloc(N * M)
    be.softmaxRowsFwdDev(ix, iy, N, M)
    assert npref.normwise(get(be, iy, N * M, (N, M)), oracle.softmax_rows(x)) < 1e-6
    dp = g.standard_normal((N, M)).astype(np.float32)
    p = oracle.softmax_rows(x)
    ip, idp, ids = put(be, p), put(be, dp), be.bufferAlloc(N * M)
    be.softmaxRowsBwdDev(ip, idp, ids, N, M)
    assert npref.normwise(get(be, ids, N * M, (N, M)), oracle.softmax_rows_bwd(p, dp)) < 1e-5
    sq = (g.standard_normal((8, 8))).astype(np.float32)
    iq = put(be, sq)
    be.causalMaskDev(iq, 8, 8, -1e9)
    ref = sq + np.triu(np.full((8, 8), -1e9, np.float32), 1)
    assert np.array_equal(get(be, iq, 64, (8, 8)), ref)


def test_invalid_handles_raise(be):
    with pytest.raises(ZillaError):
        be.reluDev(7777, 7778, 4)
    i = be.bufferAlloc(4)
    with pytest.raises(ZillaError):
        be.bufferUpload(i, np.zeros(5, np.float32))         # beyond capacity
    be.bufferFree(i)
    be.bufferFree(i)                                        # idempotent
    with pytest.raises(ZillaError):
        be.bufferDownload(i, 4)


def test_stft_and_hann(be):
    w = be.hannWindow(8)
    ref = 0.5 - 0.5 * np.cos(2 * np.pi * np.arange(8) / 7)
    np.testing.assert_allclose(w, ref, atol=1e-6)
    x = np.sin(2 * np.pi * 5 * np.arange(1024) / 64).astype(np.float32)
    mag = be.stftMagnitude(x, 64, 16)
    frames = 1 + (1024 - 64) // 16
    assert mag.shape == (33, frames)
    win = 0.5 - 0.5 * np.cos(2 * np.pi * np.arange(64) / 63)
    ref0 = np.abs(np.fft.rfft(x[:64] * win))
    np.testing.assert_allclose(mag[:, 0], ref0, atol=1e-3)


def test_softmax_ce_clamped_matches_cross_entropy_php(be):
    """softmax_ce_clamped_dev: the loss of CrossEntropy.php:56-59, -log(max(p_t, 1e-12)) per
    row, on rows with and without a target probability below 1e-12; the gradient equals
    softmax_ce_dev's (p - onehot) / B bit for bit."""
    rng = np.random.default_rng(5)
    B, C = 64, 10
    z = rng.standard_normal((B, C)).astype(np.float32)
    t = rng.integers(0, C, B).astype(np.float32)
    z[::4, :] *= 40.0                          # every fourth row: logit gaps far past 27.6
    zi, ti = put(be, z), put(be, t)
    d1, d2 = be.bufferAlloc(B * C), be.bufferAlloc(B * C)
    l1, l2 = put(be, np.zeros(1)), put(be, np.zeros(1))
    be.softmaxCeDev(zi, ti, d1, l1, B, C)
    be.softmaxCeClampedDev(zi, ti, d2, l2, B, C)
    g1, g2 = get(be, d1, B * C), get(be, d2, B * C)
    loss1, loss2 = float(get(be, l1, 1)[0]), float(get(be, l2, 1)[0])
    for i in (zi, ti, d1, d2, l1, l2):
        be.bufferFree(i)
    zz = z.astype(np.float64)
    p = np.exp(zz - zz.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    pt = p[np.arange(B), t.astype(np.int64)]
    assert (pt < 1e-12).sum() >= 4
    want = float(-np.log(np.maximum(pt, 1e-12)).sum())
    assert abs(loss2 - want) / want < 1e-5, (loss2, want)
    assert loss1 > loss2                        # the unclamped rows count more
    assert np.array_equal(g1, g2)
