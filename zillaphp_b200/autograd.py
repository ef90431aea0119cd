"""Batched autograd bridge: ZillaPHP's T1 API (Tensor -> Module -> Loss ->
Optimizer -> Trainer) over the device buffers of libzilla_b200.

The reference's autograd runs per sample on host arrays:
  - ``Tensor::conv2d`` and ``maxPool2d`` take ``[C, H, W]``
    (src/Tensor/Tensor.php:744-956);
  - every op closure is a PHP loop or a host-pointer FFI call.
Here the same methods accept a leading batch dimension (``[B, C, H, W]``;
``[C, H, W]`` still works as B = 1), and every forward and backward closure is
one call to the batched device entry points.  Values stay resident in HBM
between ops; nothing is copied to the host until ``numpy()`` / ``item()``.

Mirrors, with their semantics:
  Tensor::backward / buildTopo / accumulateGrad  src/Tensor/Tensor.php:351-387
      reverse topological order from the loss; a gradient reaching a tensor
      twice is summed (add_dev)
  Tensor::conv2d     :744-878   conv2d_batched_fwd_dev / conv2d_batched_bwd_dev
  Tensor::maxPool2d  :883-956   maxpool2d_batched_fwd_dev (argmax) / zero_dev +
                                 maxpool2d_batched_bwd_dev (scatter by argmax)
  Tensor::flatten    :958-981   a view, [B, C*H*W] (the reference's [1, N] per sample)
  Tensor::add        :1024-1032 with broadcasting of a [N] bias over [B, N] rows
                                 (add_bias_dev; reduceGrad = bias_grad_dev, :987-1022)
  Tensor::matmul     :1071-1089 matmul_dev; dA = g B^T (matmul_nt_dev), dB = A^T g (matmul_tn_dev)
  Tensor::relu       :1140-1154 relu_fwd_dev (mask) / relu_bwd_dev
  Tensor::noGrad     :54-62
  CrossEntropy       src/Loss/CrossEntropy.php:18-85: the mean over the batch of
                     -log max(p_target, 1e-12) (:58); gradient (p - onehot) / B.
                     Computed by softmax_ce_clamped_dev in fp32 (the PHP class is
                     float64), then scaled by the upstream gradient g->item() as
                     :69-70 do
  Tensor::mul        :1046-1054 mul_dev, same-shape operands only
  SGD / Adam         src/Optim/SGD.php:12-26, src/Optim/Adam.php:36-62
                     (sgd_update_dev; adam_update_dev with t counted per step)
  Conv2D / Linear / MaxPool2D / ReLU / Flatten / Sequential
                     src/NN/Layers/*.php, src/NN/Activations/ReLU.php, src/NN/Sequential.php
                     (parameters in [weight, bias] order per layer)
  Trainer::fitLoader src/Training/Trainer.php:64-98 (zeroGrad, forward, loss,
                     backward, step per batch)

Freed tensors return their buffers to a size-keyed pool that later tensors
reuse.  Every kernel runs on the library's single stream, so a buffer
handed out again is only written after its earlier readers have finished.
"""
from __future__ import annotations

import contextlib
import math

import numpy as np

from .backend import B200Backend

_BACKEND: B200Backend | None = None


def backend() -> B200Backend:
    """Tensor::backend(): the process-wide B200 backend."""
    global _BACKEND
    if _BACKEND is None:
        _BACKEND = B200Backend()
    return _BACKEND


class _Pool:
    """Device buffers by element count, recycled in stream order."""

    def __init__(self):
        self.free: dict[int, list[int]] = {}

    def get(self, n: int) -> int:
        lst = self.free.get(n)
        if lst:
            return lst.pop()
        return backend().bufferAlloc(max(n, 1))

    def put(self, n: int, buf: int) -> None:
        self.free.setdefault(n, []).append(buf)

    def clear(self) -> None:
        be = backend()
        for lst in self.free.values():
            for b in lst:
                be.bufferFree(b)
        self.free.clear()


_POOL = _Pool()
_GRAD_ENABLED = [True]


@contextlib.contextmanager
def no_grad():
    """Tensor::noGrad: no graph is recorded inside the block."""
    _GRAD_ENABLED.append(False)
    try:
        yield
    finally:
        _GRAD_ENABLED.pop()


def grad_enabled() -> bool:
    return _GRAD_ENABLED[-1]


def release_pool() -> None:
    """Frees the recycled buffers (tensors still alive keep theirs)."""
    _POOL.clear()


class Tensor:
    """A device-resident fp32 tensor with reverse-mode autograd."""

    def __init__(self, buf: int, shape, requires_grad: bool = False, base: "Tensor | None" = None):
        self.buf = buf
        self.shape = tuple(int(d) for d in shape)
        self.requires_grad = requires_grad
        self.grad: Tensor | None = None
        self.inputs: tuple = ()
        self.backward_fn = None
        self.op = "leaf"
        self._base = base            # a view keeps the tensor that owns the buffer alive
        self._pool = _POOL           # the pool (and so the backend) the buffer belongs to

    # ---------------------------------------------------------------- creation
    @classmethod
    def empty(cls, shape, requires_grad: bool = False) -> "Tensor":
        n = int(np.prod(shape)) if len(shape) else 1
        return cls(_POOL.get(n), shape, requires_grad)

    @classmethod
    def zeros(cls, shape, requires_grad: bool = False) -> "Tensor":
        t = cls.empty(shape, requires_grad)
        backend().zeroDev(t.buf, t.size)
        return t

    @classmethod
    def from_numpy(cls, a, requires_grad: bool = False) -> "Tensor":
        a = np.ascontiguousarray(a, np.float32)
        t = cls.empty(a.shape if a.ndim else (1,), requires_grad)
        backend().bufferUpload(t.buf, a)
        return t

    def __del__(self):
        try:
            if self._base is None and self.buf > 0:
                self._pool.put(self.size, self.buf)
                self.buf = 0
        except Exception:  # noqa: BLE001 (interpreter shutdown)
            pass

    # ---------------------------------------------------------------- access
    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if len(self.shape) else 1

    def numpy(self) -> np.ndarray:
        return backend().bufferDownload(self.buf, self.size).reshape(self.shape)

    def item(self) -> float:
        return float(backend().bufferDownload(self.buf, 1)[0])

    def zero_grad(self) -> None:
        self.grad = None

    def view(self, shape) -> "Tensor":
        assert int(np.prod(shape)) == self.size
        return Tensor(self.buf, shape, False, self._base or self)

    # ---------------------------------------------------------------- autograd
    def _attach(self, inputs, op: str, fn) -> "Tensor":
        if grad_enabled() and any(i.requires_grad for i in inputs):
            self.requires_grad = True
            self.inputs = tuple(inputs)
            self.op = op
            self.backward_fn = fn
        return self

    def accumulate_grad(self, g: "Tensor") -> None:
        """accumulateGrad: the first gradient is taken over, later ones summed."""
        if self.grad is None:
            self.grad = g if g.shape == self.shape else g.view(self.shape)
        else:
            backend().addDev(self.grad.buf, g.buf, self.grad.buf, self.size)

    def backward(self) -> None:
        """Tensor::backward on a scalar loss (seed gradient 1)."""
        order, seen = [], set()
        stack = [(self, False)]
        while stack:   # iterative post-order DFS (buildTopo)
            t, done = stack.pop()
            if done:
                order.append(t)
                continue
            if id(t) in seen:
                continue
            seen.add(id(t))
            stack.append((t, True))
            for i in t.inputs:
                if i.requires_grad and id(i) not in seen:
                    stack.append((i, False))
        if self.grad is None:
            self.grad = Tensor.from_numpy(np.ones(self.shape, np.float32))
            self.grad.seed_one = True   # known to be 1 on the host: no device read needed
        for t in reversed(order):
            if t.backward_fn is not None and t.grad is not None:
                t.backward_fn(t.grad)

    # ---------------------------------------------------------------- ops
    def conv2d(self, weight: "Tensor", bias: "Tensor", stride: int = 1, padding: int = 0) -> "Tensor":
        squeeze = len(self.shape) == 3
        B, C, H, W = (1,) + self.shape if squeeze else self.shape
        if len(weight.shape) != 4:
            raise RuntimeError("conv2d weight must be [outC, C, kH, kW].")
        oC, Cw, kH, kW = weight.shape
        if Cw != C:
            raise ValueError(f"conv2d: channel mismatch ({C} vs {Cw}).")
        oH, oW = (H + 2 * padding - kH) // stride + 1, (W + 2 * padding - kW) // stride + 1
        out_shape = (oC, oH, oW) if squeeze else (B, oC, oH, oW)
        out = Tensor.empty(out_shape)
        be = backend()
        be.conv2dBatchedFwdDev(self.buf, weight.buf, bias.buf, out.buf, B, C, H, W, oC, oH, oW, kH, kW,
                               stride, padding)
        x = self

        def fn(g: Tensor) -> None:
            gi, gw, gb = Tensor.empty(x.shape), Tensor.empty(weight.shape), Tensor.empty(bias.shape)
            be.conv2dBatchedBwdDev(x.buf, weight.buf, g.buf, gi.buf, gw.buf, gb.buf, B, C, H, W, oC, oH, oW,
                                   kH, kW, stride, padding)
            if x.requires_grad:
                x.accumulate_grad(gi)
            if weight.requires_grad:
                weight.accumulate_grad(gw)
            if bias.requires_grad:
                bias.accumulate_grad(gb)

        return out._attach((self, weight, bias), "conv2d", fn)

    def maxPool2d(self, kernelSize: int, stride: int | None = None) -> "Tensor":  # noqa: N802,N803
        stride = kernelSize if stride is None else stride
        squeeze = len(self.shape) == 3
        B, C, H, W = (1,) + self.shape if squeeze else self.shape
        oH, oW = (H - kernelSize) // stride + 1, (W - kernelSize) // stride + 1
        out = Tensor.empty((C, oH, oW) if squeeze else (B, C, oH, oW))
        arg = Tensor.empty(out.shape)          # int32 indices in a float buffer
        be = backend()
        be.maxPool2dBatchedFwdDev(self.buf, out.buf, arg.buf, B, C, H, W, oH, oW, kernelSize, kernelSize, stride)
        out.argmax = arg
        x = self

        def fn(g: Tensor) -> None:
            gi = Tensor.zeros(x.shape)         # the scatter adds into a zeroed input gradient
            be.maxPool2dBatchedBwdDev(g.buf, arg.buf, gi.buf, B, C, oH, oW)
            x.accumulate_grad(gi)

        return out._attach((self,), "maxPool2d", fn)

    def relu(self) -> "Tensor":
        out, mask = Tensor.empty(self.shape), Tensor.empty(self.shape)
        be = backend()
        be.reluFwdDev(self.buf, out.buf, mask.buf, self.size)
        x = self

        def fn(g: Tensor) -> None:
            gi = Tensor.empty(x.shape)
            be.reluBwdDev(g.buf, mask.buf, gi.buf, x.size)
            x.accumulate_grad(gi)

        return out._attach((self,), "relu", fn)

    def flatten(self) -> "Tensor":
        """[B, C, H, W] -> [B, C*H*W] (NCHW order); [C, H, W] -> [1, C*H*W] as the reference."""
        rows = self.shape[0] if len(self.shape) == 4 else 1
        out = self.view((rows, self.size // rows))
        out.requires_grad = False
        x = self

        def fn(g: Tensor) -> None:
            x.accumulate_grad(g.view(x.shape))

        return out._attach((self,), "flatten", fn)

    def matmul(self, other: "Tensor") -> "Tensor":
        M, K = self.shape
        K2, N = other.shape
        if K != K2:
            raise ValueError(f"matmul: inner dimensions differ ({K} vs {K2}).")
        out = Tensor.empty((M, N))
        be = backend()
        be.matmulDev(self.buf, other.buf, out.buf, M, K, N)
        a, b = self, other

        def fn(g: Tensor) -> None:
            if a.requires_grad:
                ga = Tensor.empty((M, K))
                be.matmulNtDev(g.buf, b.buf, ga.buf, M, N, K)     # g [M,N] . B^T, B stored [K,N]
                a.accumulate_grad(ga)
            if b.requires_grad:
                gb = Tensor.empty((K, N))
                be.matmulTnDev(a.buf, g.buf, gb.buf, K, M, N)     # A^T [K,M] . g [M,N], A stored [M,K]
                b.accumulate_grad(gb)

        return out._attach((self, other), "matmul", fn)

    def add(self, other: "Tensor") -> "Tensor":
        """Elementwise sum; a 1-D [N] operand broadcasts over the rows of [B, N]."""
        be = backend()
        out = Tensor.empty(self.shape)
        if other.shape == self.shape:
            be.addDev(self.buf, other.buf, out.buf, self.size)
            bias_rows = 0
        elif len(other.shape) == 1 and self.shape[-1] == other.shape[0]:
            bias_rows = self.size // other.shape[0]
            be.copyDev(self.buf, out.buf, self.size)
            be.addBiasDev(out.buf, other.buf, bias_rows, other.shape[0])
        else:
            raise ValueError(f"add: cannot broadcast {other.shape} onto {self.shape}.")
        a, b = self, other

        def fn(g: Tensor) -> None:
            if b.requires_grad:
                if bias_rows:
                    gb = Tensor.empty(b.shape)
                    be.biasGradDev(g.buf, gb.buf, bias_rows, b.shape[0])   # reduceGrad: sum over rows
                    b.accumulate_grad(gb)
                elif a.requires_grad and a is not b:   # both keep g: b gets its own copy
                    gb = Tensor.empty(b.shape)
                    be.copyDev(g.buf, gb.buf, b.size)
                    b.accumulate_grad(gb)
                else:
                    b.accumulate_grad(g)
            if a.requires_grad:
                a.accumulate_grad(g)

        return out._attach((self, other), "add", fn)


    def mul(self, other: "Tensor") -> "Tensor":
        """Elementwise product of two tensors of the same shape (Tensor::mul, :1046-1054, without
        broadcasting): dA = g * B, dB = g * A."""
        if other.shape != self.shape:
            raise ValueError(f"mul: shapes {self.shape} and {other.shape} differ.")
        be = backend()
        out = Tensor.empty(self.shape)
        be.mulDev(self.buf, other.buf, out.buf, self.size)
        a, b = self, other

        def fn(g: Tensor) -> None:
            if a.requires_grad:
                ga = Tensor.empty(a.shape)
                be.mulDev(g.buf, b.buf, ga.buf, a.size)
                a.accumulate_grad(ga)
            if b.requires_grad:
                gb = Tensor.empty(b.shape)
                be.mulDev(g.buf, a.buf, gb.buf, b.size)
                b.accumulate_grad(gb)

        return out._attach((self, other), "mul", fn)


class Parameter(Tensor):
    """src/NN/Parameter.php: a leaf tensor that requires gradients."""

    def __init__(self, data: np.ndarray):
        a = np.ascontiguousarray(data, np.float32)
        super().__init__(_POOL.get(a.size), a.shape, True)
        backend().bufferUpload(self.buf, a)

    def load(self, data: np.ndarray) -> None:
        a = np.ascontiguousarray(data, np.float32).reshape(self.shape)
        backend().bufferUpload(self.buf, a)


# -------------------------------------------------------------------- modules
class Module:
    def forward(self, x: Tensor) -> Tensor:
        raise NotImplementedError

    def __call__(self, x: Tensor) -> Tensor:
        return self.forward(x)

    def parameters(self) -> list[Parameter]:
        return []


class Conv2D(Module):
    """src/NN/Layers/Conv2D.php: weight [outC, inC, k, k] (He normal), bias zeros."""

    def __init__(self, inChannels: int, outChannels: int, kernelSize: int = 3, stride: int = 1,  # noqa: N803
                 padding: int = 0, rng: np.random.Generator | None = None):
        rng = rng or np.random.default_rng(0)
        std = math.sqrt(2.0 / max(inChannels * kernelSize * kernelSize, 1))
        self.weight = Parameter(rng.standard_normal((outChannels, inChannels, kernelSize, kernelSize)) * std)
        self.bias = Parameter(np.zeros(outChannels))
        self.stride, self.padding = stride, padding

    def forward(self, x: Tensor) -> Tensor:
        return x.conv2d(self.weight, self.bias, self.stride, self.padding)

    def parameters(self) -> list[Parameter]:
        return [self.weight, self.bias]


class Linear(Module):
    """src/NN/Layers/Linear.php: weight [in, out] ~ N(0, 1/in), bias zeros; x W then + b."""

    def __init__(self, inFeatures: int, outFeatures: int, rng: np.random.Generator | None = None):  # noqa: N803
        rng = rng or np.random.default_rng(0)
        self.weight = Parameter(rng.standard_normal((inFeatures, outFeatures)) * math.sqrt(1.0 / max(inFeatures, 1)))
        self.bias = Parameter(np.zeros(outFeatures))

    def forward(self, x: Tensor) -> Tensor:
        return x.matmul(self.weight).add(self.bias)

    def parameters(self) -> list[Parameter]:
        return [self.weight, self.bias]


class MaxPool2D(Module):
    def __init__(self, kernelSize: int = 2, stride: int | None = None):  # noqa: N803
        self.k, self.stride = kernelSize, stride

    def forward(self, x: Tensor) -> Tensor:
        return x.maxPool2d(self.k, self.stride)


class ReLU(Module):
    def forward(self, x: Tensor) -> Tensor:
        return x.relu()


class Flatten(Module):
    def forward(self, x: Tensor) -> Tensor:
        return x.flatten()


class Sequential(Module):
    """src/NN/Sequential.php: layers in order; parameters() concatenated in layer order."""

    def __init__(self, *layers: Module):
        self.layers = list(layers)

    def forward(self, x: Tensor) -> Tensor:
        for layer in self.layers:
            x = layer(x)
        return x

    def parameters(self) -> list[Parameter]:
        return [p for layer in self.layers for p in layer.parameters()]

    def load_flat(self, flat: np.ndarray) -> None:
        """Sets every parameter from one flat vector in parameters() order."""
        off = 0
        for p in self.parameters():
            p.load(flat[off:off + p.size])
            off += p.size
        assert off == flat.size, (off, flat.size)

    def flat(self, grads: bool = False) -> np.ndarray:
        parts = []
        for p in self.parameters():
            t = p.grad if grads else p
            parts.append(t.numpy().ravel() if t is not None else np.zeros(p.size, np.float32))
        return np.concatenate(parts)


# -------------------------------------------------------------------- loss
class CrossEntropy:
    """src/Loss/CrossEntropy.php: mean over the batch of -log softmax(pred)[target]."""

    def forward(self, pred: Tensor, targets) -> Tensor:
        B, Cn = pred.shape
        y = targets if isinstance(targets, Tensor) else Tensor.from_numpy(np.asarray(targets, np.float32).reshape(B))
        dlogits = Tensor.empty((B, Cn))
        loss = Tensor.zeros((1,))
        be = backend()
        be.softmaxCeClampedDev(pred.buf, y.buf, dlogits.buf, loss.buf, B, Cn)   # loss SUM (p_t >= 1e-12), dlogits = (p - 1hot)/B
        be.scaleDev(loss.buf, 1.0 / B, 1)                                  # the mean
        p = pred

        def fn(g: Tensor) -> None:
            # CrossEntropy.php:69-70: the gradient is (p - onehot) * g->item() / batch.  The seed
            # gradient of a loss that is the root of backward() is 1 and needs no device read.
            s = 1.0 if getattr(g, "seed_one", False) else float(g.item())
            if s == 1.0:
                p.accumulate_grad(dlogits)
                return
            scaled = Tensor.empty(dlogits.shape)
            be.copyDev(dlogits.buf, scaled.buf, dlogits.size)
            be.scaleDev(scaled.buf, s, scaled.size)
            p.accumulate_grad(scaled)

        return loss._attach((pred,), "cross_entropy", fn)

    __call__ = forward


# -------------------------------------------------------------------- optimizers
class SGD:
    """src/Optim/SGD.php: w -= lr * grad."""

    def __init__(self, params: list[Parameter], lr: float = 0.01):
        self.params, self.lr = list(params), lr

    def zeroGrad(self) -> None:  # noqa: N802
        for p in self.params:
            p.grad = None

    def step(self) -> None:
        be = backend()
        for p in self.params:
            if p.grad is not None:
                be.sgdUpdateDev(p.buf, p.grad.buf, self.lr, p.size)


class Adam:
    """src/Optim/Adam.php: bias-corrected moments, t incremented once per step."""

    def __init__(self, params: list[Parameter], lr: float = 1e-3, beta1: float = 0.9, beta2: float = 0.999,
                 eps: float = 1e-8):
        self.params = list(params)
        self.lr, self.b1, self.b2, self.eps = lr, beta1, beta2, eps
        self.t = 0
        self.m = [Tensor.zeros(p.shape) for p in self.params]
        self.v = [Tensor.zeros(p.shape) for p in self.params]

    def zeroGrad(self) -> None:  # noqa: N802
        for p in self.params:
            p.grad = None

    def step(self) -> None:
        self.t += 1
        be = backend()
        for p, m, v in zip(self.params, self.m, self.v):
            if p.grad is not None:
                be.adamUpdateDev(p.buf, p.grad.buf, m.buf, v.buf, self.lr, self.b1, self.b2, self.eps, self.t,
                                 p.size)


# -------------------------------------------------------------------- trainer
class Trainer:
    """src/Training/Trainer.php fitLoader: per batch zeroGrad, forward, loss,
    backward, step; returns the mean of the batches' losses per epoch."""

    def __init__(self, model: Module, optimizer, loss):
        self.model, self.optimizer, self.loss = model, optimizer, loss

    def step(self, x: np.ndarray | Tensor, y) -> float:
        xt = x if isinstance(x, Tensor) else Tensor.from_numpy(x)
        self.optimizer.zeroGrad()
        pred = self.model.forward(xt)
        loss = self.loss.forward(pred, y)
        loss.backward()
        self.optimizer.step()
        return loss.item()

    def fitLoader(self, batches, epochs: int = 1, onEpoch=None) -> list[float]:  # noqa: N802,N803
        history = []
        for epoch in range(epochs):
            total, n = 0.0, 0
            for x, y in batches:
                total += self.step(x, y)
                n += 1
            avg = total / max(n, 1)
            history.append(avg)
            if onEpoch is not None:
                onEpoch(epoch, avg)
        return history


def sequential_from_spec(layers, in_shape, rng: np.random.Generator | None = None) -> Sequential:
    """A Sequential from the fused step's layer rows {kind, a, b, c}
    (1 Conv2D 3x3 (in, out, padding), 2 ReLU, 3 MaxPool2D 2x2, 4 Linear (in, out)),
    with a Flatten before the first Linear that follows a [C, H, W] activation."""
    from .configs import CONV, LINEAR, POOL, RELU
    rng = rng or np.random.default_rng(0)
    mods: list[Module] = []
    spatial = len(in_shape) == 3 and not (in_shape[1] == 1 and in_shape[2] == 1)
    first = True
    for kind, a, b, c in layers:
        if kind == CONV:
            mods.append(Conv2D(a, b, 3, 1, c, rng))
            spatial = True
        elif kind == RELU:
            mods.append(ReLU())
        elif kind == POOL:
            mods.append(MaxPool2D(2))
        elif kind == LINEAR:
            if spatial or first:
                mods.append(Flatten())
                spatial = False
            mods.append(Linear(a, b, rng))
        else:
            raise ValueError(f"unknown layer kind {kind}")
        first = False
    return Sequential(*mods)
