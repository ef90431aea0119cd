"""The B200Backend device-op surface on host arrays, each op computed by the
oracle (test infrastructure): lets the autograd bridge's wiring (graph order,
gradient accumulation, broadcasting, optimizer bookkeeping) run on the CPU.
Buffers are float32 numpy arrays keyed by handle, as in the registry."""
import numpy as np

import oracle


class OracleBackend:
    def __init__(self):
        self.bufs: dict[int, np.ndarray] = {}
        self.next = 1
        self.calls: list[str] = []

    def _b(self, i, n, shape=None):
        a = self.bufs[i][:n]
        return a.reshape(shape) if shape is not None else a

    # registry
    def bufferAlloc(self, n):  # noqa: N802
        i = self.next
        self.next += 1
        self.bufs[i] = np.zeros(n, np.float32)
        return i

    def bufferFree(self, i):  # noqa: N802
        self.bufs.pop(i, None)

    def bufferUpload(self, i, host):  # noqa: N802
        a = np.ascontiguousarray(host, np.float32).ravel()
        self.bufs[i][:a.size] = a

    def bufferDownload(self, i, n):  # noqa: N802
        return self.bufs[i][:n].copy()

    # elementwise
    def zeroDev(self, i, n):  # noqa: N802
        self.bufs[i][:n] = 0.0

    def copyDev(self, s, d, n):  # noqa: N802
        self.bufs[d][:n] = self.bufs[s][:n]

    def addDev(self, a, b, c, n):  # noqa: N802
        self.bufs[c][:n] = self.bufs[a][:n] + self.bufs[b][:n]

    def mulDev(self, a, b, c, n):  # noqa: N802
        self.bufs[c][:n] = self.bufs[a][:n] * self.bufs[b][:n]

    def scaleDev(self, x, s, n):  # noqa: N802
        self.bufs[x][:n] *= np.float32(s)

    # conv / pool
    def conv2dBatchedFwdDev(self, i, w, b, o, B, C, H, W, oC, oH, oW, kH, kW, s, p):  # noqa: N802
        self.calls.append("conv2d_batched_fwd_dev")
        y = oracle.conv2d_batched_forward(self._b(i, B * C * H * W, (B, C, H, W)),
                                          self._b(w, oC * C * kH * kW, (oC, C, kH, kW)), self._b(b, oC), s, p)
        self.bufs[o][:y.size] = y.ravel()

    def conv2dBatchedBwdDev(self, i, w, go, gi, gw, gb, B, C, H, W, oC, oH, oW, kH, kW, s, p):  # noqa: N802
        self.calls.append("conv2d_batched_bwd_dev")
        dx, dw, db = oracle.conv2d_batched_backward(self._b(i, B * C * H * W, (B, C, H, W)),
                                                    self._b(w, oC * C * kH * kW, (oC, C, kH, kW)),
                                                    self._b(go, B * oC * oH * oW, (B, oC, oH, oW)), s, p)
        self.bufs[gi][:dx.size] = dx.ravel()
        self.bufs[gw][:dw.size] = dw.ravel()
        self.bufs[gb][:db.size] = db

    def maxPool2dBatchedFwdDev(self, i, o, a, B, C, H, W, oH, oW, kH, kW, s):  # noqa: N802
        self.calls.append("maxpool2d_batched_fwd_dev")
        y, am = oracle.maxpool2d_batched_forward(self._b(i, B * C * H * W, (B, C, H, W)), kH, s)
        self.bufs[o][:y.size] = y.ravel()
        self.bufs[a][:am.size] = am.ravel().view(np.float32)

    def maxPool2dBatchedBwdDev(self, go, a, gi, B, C, oH, oW):  # noqa: N802
        self.calls.append("maxpool2d_batched_bwd_dev")
        n = B * C * oH * oW
        idx = self.bufs[a][:n].view(np.int32)
        np.add.at(self.bufs[gi], idx, self.bufs[go][:n])

    # training ops
    def reluFwdDev(self, x, y, m, n):  # noqa: N802
        out, mask = oracle.relu_fwd_dev(self._b(x, n))
        self.bufs[y][:n] = out
        self.bufs[m][:n] = mask

    def reluBwdDev(self, dy, m, dx, n):  # noqa: N802
        self.bufs[dx][:n] = oracle.relu_bwd_dev(self._b(dy, n), self._b(m, n))

    def matmulDev(self, a, b, c, M, K, N):  # noqa: N802
        self.bufs[c][:M * N] = oracle.matmul_dev(self._b(a, M * K, (M, K)), self._b(b, K * N, (K, N)), "nn").ravel()

    def matmulNtDev(self, a, b, c, M, K, N):  # noqa: N802
        self.bufs[c][:M * N] = oracle.matmul_dev(self._b(a, M * K, (M, K)), self._b(b, N * K, (N, K)), "nt").ravel()

    def matmulTnDev(self, a, b, c, M, K, N):  # noqa: N802
        self.bufs[c][:M * N] = oracle.matmul_dev(self._b(a, K * M, (K, M)), self._b(b, K * N, (K, N)), "tn").ravel()

    def addBiasDev(self, x, b, B, C):  # noqa: N802
        self.bufs[x][:B * C] = oracle.add_bias_dev(self._b(x, B * C, (B, C)), self._b(b, C)).ravel()

    def biasGradDev(self, dy, db, B, C):  # noqa: N802
        self.bufs[db][:C] = oracle.bias_grad_dev(self._b(dy, B * C, (B, C)))

    def softmaxCeDev(self, z, t, dl, loss, B, C):  # noqa: N802
        g, s = oracle.softmax_ce_dev(self._b(z, B * C, (B, C)), self._b(t, B), loss0=float(self.bufs[loss][0]))
        self.bufs[dl][:B * C] = g.ravel()
        self.bufs[loss][0] = s

    def softmaxCeClampedDev(self, z, t, dl, loss, B, C):  # noqa: N802
        """CrossEntropy.php:56-59 in float64: the rows' -log(max(p_t, 1e-12)); softmax_ce_dev's gradient."""
        zz = self._b(z, B * C, (B, C)).astype(np.float64)
        tt = self._b(t, B).astype(np.int64)
        g, _ = oracle.softmax_ce_dev(self._b(z, B * C, (B, C)), self._b(t, B), loss0=0.0)
        p = np.exp(zz - zz.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        self.bufs[dl][:B * C] = g.ravel()
        self.bufs[loss][0] = np.float32(float(self.bufs[loss][0]) + float(-np.log(np.maximum(p[np.arange(B), tt], 1e-12)).sum()))

    def sgdUpdateDev(self, w, g, lr, n):  # noqa: N802
        self.bufs[w][:n] = oracle.sgd_update_dev(self._b(w, n), self._b(g, n), lr)

    def adamUpdateDev(self, w, g, m, v, lr, b1, b2, eps, t, n):  # noqa: N802
        nw, nm, nv = oracle.adam_update(self._b(w, n), self._b(g, n), self._b(m, n), self._b(v, n), lr, b1, b2, eps, t)
        self.bufs[w][:n], self.bufs[m][:n], self.bufs[v][:n] = nw, nm, nv
