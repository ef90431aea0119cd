"""CPU oracle for the ZillaPHP training hot path (TEST INFRASTRUCTURE ONLY).

Only tests, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module, and only as the checker / the timed
reference CPU run.  The product never routes through it.

Three shared libraries are reachable from here:

* ``lib/libzilla_oracle.so`` -- the C restatement in ``zilla_oracle.c`` plus
  the step driver ``cnn_step.c`` (strict IEEE build).  Default checker.
* ``_ref/libzilla_cpu_ref_strict.so`` -- the reference CPU library
  (native/cpu/*.c) compiled from its own sources with strict flags; used to
  pin the restatement.
* ``_ref/libzilla_refstep.so`` -- the step driver linked against the
  reference CPU library built with its own flags and OpenBLAS: the timed
  reference CPU baseline.

The op wrappers below take and return numpy arrays and hide the handle
registry of the reference ABI (native/cpu/buffer_registry.c:16-88).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBS = {
    "oracle": os.path.join(HERE, "lib", "libzilla_oracle.so"),
    "ref_strict": os.path.join(HERE, "_ref", "libzilla_cpu_ref_strict.so"),
    "ref": os.path.join(HERE, "_ref", "libzilla_cpu_ref.so"),
    "refstep": os.path.join(HERE, "_ref", "libzilla_refstep.so"),
}

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_cache: dict[str, C.CDLL] = {}


def build() -> None:
    """Compile the oracle (and, where the reference sources exist, _ref/)."""
    subprocess.run(["make", "-s", "-C", HERE, f"PYTHON={os.sys.executable}"], check=True)


def available(kind: str) -> bool:
    return os.path.exists(LIBS[kind])


def lib(kind: str = "oracle") -> C.CDLL:
    if kind in _cache:
        return _cache[kind]
    path = LIBS[kind]
    if not os.path.exists(path):
        raise FileNotFoundError(f"oracle library {path} not built (run make -C oracle)")
    L = C.CDLL(path)
    if kind in ("oracle", "ref_strict", "ref"):
        L.zilla_cpu_buffer_alloc.restype = C.c_int
        L.zilla_cpu_buffer_alloc.argtypes = [C.c_size_t]
        L.zilla_cpu_buffer_ptr.restype = C.POINTER(C.c_float)
        L.zilla_cpu_buffer_ptr.argtypes = [C.c_int]
        L.zilla_cpu_buffer_upload.argtypes = [C.c_int, _f32p, C.c_size_t]
        L.zilla_cpu_buffer_download.argtypes = [C.c_int, _f32p, C.c_size_t]
        L.zilla_cpu_buffer_free.argtypes = [C.c_int]
        L.conv2d_forward_f32.argtypes = [_f32p, _f32p, _f32p, _f32p] + [C.c_int] * 8
        L.conv2d_backward_f32.argtypes = [_f32p] * 6 + [C.c_int] * 8
        L.maxpool2d_forward_f32.argtypes = [_f32p, _f32p, _i32p] + [C.c_int] * 6
        L.maxpool2d_backward_f32.argtypes = [_f32p, _i32p, _f32p] + [C.c_int] * 5
        L.matmul_f32.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int]
        L.sgd_update_dev.argtypes = [C.c_int, C.c_int, C.c_float, C.c_int]
    if kind == "oracle":
        L.oracle_adam_update.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_long,
                                         C.c_double, C.c_double, C.c_double, C.c_double, C.c_int]
        L.oracle_maxpool_batched_fwd.argtypes = [_f32p, _f32p, _i32p] + [C.c_int] * 7
        L.oracle_softmax_rows.argtypes = [_f32p, _f32p, C.c_int, C.c_int]
        L.oracle_softmax_rows_bwd.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int]
        L.oracle_cross_entropy_mean.restype = C.c_double
        L.oracle_cross_entropy_mean.argtypes = [_f32p, _i32p, _f32p, C.c_int, C.c_int]
    if kind in ("oracle", "refstep"):
        L.zo_model_create.restype = C.c_void_p
        L.zo_model_create.argtypes = [_i32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        L.zo_model_destroy.argtypes = [C.c_void_p]
        L.zo_model_nparams.restype = C.c_long
        L.zo_model_nparams.argtypes = [C.c_void_p]
        for fn in ("zo_model_params", "zo_model_grads", "zo_model_dlogits"):
            getattr(L, fn).restype = C.POINTER(C.c_float)
            getattr(L, fn).argtypes = [C.c_void_p]
        L.zo_model_output.restype = C.POINTER(C.c_float)
        L.zo_model_output.argtypes = [C.c_void_p, C.c_int]
        L.zo_model_argmax.restype = C.POINTER(C.c_int)
        L.zo_model_argmax.argtypes = [C.c_void_p, C.c_int]
        L.zo_model_step.restype = C.c_int
        L.zo_model_step.argtypes = [C.c_void_p, _f32p, _f32p, C.c_int, C.c_float,
                                    C.POINTER(C.c_float)]
    _cache[kind] = L
    return L


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------- handles
class _Reg:
    """Scoped registry buffers of one oracle library."""

    def __init__(self, L):
        self.L, self.ids = L, []

    def put(self, a) -> int:
        a = _f32(a).ravel()
        i = self.L.zilla_cpu_buffer_alloc(max(a.size, 1))
        assert i > 0
        if a.size:
            self.L.zilla_cpu_buffer_upload(i, a, a.size)
        self.ids.append(i)
        return i

    def new(self, n: int) -> int:
        return self.put(np.zeros(n, np.float32))

    def get(self, i: int, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        self.L.zilla_cpu_buffer_download(i, out, n)
        return out

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        for i in self.ids:
            self.L.zilla_cpu_buffer_free(i)


# ---------------------------------------------------------------- host-pointer ops
def conv2d_forward(x, w, b, stride=1, pad=0, kind="oracle"):
    """native/cpu/zilla_cpu.c:112-145 on one sample x[C,H,W]."""
    L = lib(kind)
    x, w, b = _f32(x), _f32(w), _f32(b)
    Cin, H, W = x.shape
    Co, _, kh, kw = w.shape
    oH, oW = (H + 2 * pad - kh) // stride + 1, (W + 2 * pad - kw) // stride + 1
    out = np.empty((Co, oH, oW), np.float32)
    L.conv2d_forward_f32(x, w, b, out, Cin, H, W, Co, kh, kw, stride, pad)
    return out


def conv2d_backward(x, w, gout, stride=1, pad=0, kind="oracle"):
    """native/cpu/zilla_cpu.c:147-195 on one sample; returns (dx, dw, db)."""
    L = lib(kind)
    x, w, gout = _f32(x), _f32(w), _f32(gout)
    Cin, H, W = x.shape
    Co, _, kh, kw = w.shape
    gi = np.empty_like(x)
    gw = np.empty_like(w)
    gb = np.empty(Co, np.float32)
    L.conv2d_backward_f32(x, w, gout, gi, gw, gb, Cin, H, W, Co, kh, kw, stride, pad)
    return gi, gw, gb


def conv2d_batched_forward(x, w, b, stride=1, pad=0, kind="oracle"):
    return np.stack([conv2d_forward(xi, w, b, stride, pad, kind) for xi in x])


def conv2d_batched_backward(x, w, gout, stride=1, pad=0, kind="oracle"):
    """Per-sample backward looped over the batch; dW and db summed in sample order."""
    gis, gw, gb = [], None, None
    for xi, gi in zip(x, gout):
        a, bw, bb = conv2d_backward(xi, w, gi, stride, pad, kind)
        gis.append(a)
        gw = bw.copy() if gw is None else (gw + bw).astype(np.float32)
        gb = bb.copy() if gb is None else (gb + bb).astype(np.float32)
    return np.stack(gis), gw, gb


def maxpool2d_forward(x, k=2, stride=2, kind="oracle"):
    """native/cpu/zilla_cpu.c:201-232 on x[C,H,W]; argmax channel-local."""
    L = lib(kind)
    x = _f32(x)
    Cn, H, W = x.shape
    oH, oW = (H - k) // stride + 1, (W - k) // stride + 1
    out = np.empty((Cn, oH, oW), np.float32)
    am = np.empty((Cn, oH, oW), np.int32)
    L.maxpool2d_forward_f32(x, out, am, Cn, H, W, k, k, stride)
    return out, am


def maxpool2d_batched_forward(x, k=2, stride=2):
    """Batched pool with the GPU batched argmax convention (flat index into [B,C,H,W])."""
    L = lib("oracle")
    x = _f32(x)
    B, Cn, H, W = x.shape
    oH, oW = (H - k) // stride + 1, (W - k) // stride + 1
    out = np.empty((B, Cn, oH, oW), np.float32)
    am = np.empty((B, Cn, oH, oW), np.int32)
    L.oracle_maxpool_batched_fwd(x, out, am, B, Cn, H, W, k, k, stride)
    return out, am


def maxpool2d_backward(gout, argmax, H, W, kind="oracle"):
    """native/cpu/zilla_cpu.c:234-251 on one sample (channel-local argmax)."""
    L = lib(kind)
    gout = _f32(gout)
    argmax = np.ascontiguousarray(argmax, np.int32)
    Cn, oH, oW = gout.shape
    gi = np.empty((Cn, H, W), np.float32)
    L.maxpool2d_backward_f32(gout, argmax, gi, Cn, H, W, oH, oW)
    return gi


def matmul(a, b, kind="oracle"):
    """native/cpu/zilla_cpu.c:27-64 (host pointer)."""
    L = lib(kind)
    a, b = _f32(a), _f32(b)
    out = np.empty((a.shape[0], b.shape[1]), np.float32)
    L.matmul_f32(a, b, out, a.shape[0], a.shape[1], b.shape[1])
    return out


# ---------------------------------------------------------------- handle ops
def matmul_dev(a, b, variant="nn", kind="oracle"):
    """native/cpu/training_ops.c:25-105: nn C=A@B, tn C=A^T@B (A [K,M]), nt C=A@B^T (B [N,K])."""
    L = lib(kind)
    a, b = _f32(a), _f32(b)
    if variant == "nn":
        M, K = a.shape; N = b.shape[1]
    elif variant == "tn":
        K, M = a.shape; N = b.shape[1]
    else:
        M, K = a.shape; N = b.shape[0]
    fn = {"nn": L.matmul_dev, "tn": L.matmul_tn_dev, "nt": L.matmul_nt_dev}[variant]
    with _Reg(L) as R:
        ia, ib, ic = R.put(a), R.put(b), R.new(M * N)
        assert fn(ia, ib, ic, M, K, N) == 0
        return R.get(ic, M * N).reshape(M, N)


def add_bias_dev(x, b, kind="oracle"):
    L = lib(kind)
    x = _f32(x)
    with _Reg(L) as R:
        ix, ib = R.put(x), R.put(b)
        assert L.add_bias_dev(ix, ib, x.shape[0], x.shape[1]) == 0
        return R.get(ix, x.size).reshape(x.shape)


def relu_fwd_dev(x, kind="oracle"):
    L = lib(kind)
    x = _f32(x)
    with _Reg(L) as R:
        ix, iy, im = R.put(x), R.new(x.size), R.new(x.size)
        assert L.relu_fwd_dev(ix, iy, im, x.size) == 0
        return R.get(iy, x.size).reshape(x.shape), R.get(im, x.size).reshape(x.shape)


def relu_bwd_dev(dy, mask, kind="oracle"):
    L = lib(kind)
    dy = _f32(dy)
    with _Reg(L) as R:
        a, m, o = R.put(dy), R.put(mask), R.new(dy.size)
        assert L.relu_bwd_dev(a, m, o, dy.size) == 0
        return R.get(o, dy.size).reshape(dy.shape)


def softmax_ce_dev(logits, targets, loss0=0.0, kind="oracle"):
    """native/cpu/training_ops.c:162-206: returns (dlogits, loss_sum) or rc for errors."""
    L = lib(kind)
    z = _f32(logits)
    B, Cn = z.shape
    with _Reg(L) as R:
        iz, it, idl, il = R.put(z), R.put(np.asarray(targets, np.float32)), R.new(z.size), R.put([loss0])
        rc = L.softmax_ce_dev(iz, it, idl, il, B, Cn)
        if rc:
            return rc
        return R.get(idl, z.size).reshape(B, Cn), float(R.get(il, 1)[0])


def bias_grad_dev(dy, kind="oracle"):
    L = lib(kind)
    dy = _f32(dy)
    with _Reg(L) as R:
        a, o = R.put(dy), R.new(dy.shape[1])
        assert L.bias_grad_dev(a, o, dy.shape[0], dy.shape[1]) == 0
        return R.get(o, dy.shape[1])


def sgd_update_dev(w, g, lr, kind="oracle"):
    L = lib(kind)
    w = _f32(w)
    with _Reg(L) as R:
        iw, ig = R.put(w), R.put(g)
        assert L.sgd_update_dev(iw, ig, lr, w.size) == 0
        return R.get(iw, w.size).reshape(w.shape)


def adam_update(w, g, m, v, lr, b1=0.9, b2=0.999, eps=1e-8, t=1):
    """src/Optim/Adam.php:36-62 restated (float buffers, double arithmetic)."""
    w, g, m, v = (_f32(a).copy() for a in (w, g, m, v))
    lib("oracle").oracle_adam_update(w, g, m, v, w.size, lr, b1, b2, eps, t)
    return w, m, v


def softmax_rows(x):
    x = _f32(x)
    y = np.empty_like(x)
    lib("oracle").oracle_softmax_rows(x, y, x.shape[0], x.shape[1])
    return y


def softmax_rows_bwd(P, dP):
    P, dP = _f32(P), _f32(dP)
    dS = np.empty_like(P)
    lib("oracle").oracle_softmax_rows_bwd(P, dP, dS, P.shape[0], P.shape[1])
    return dS


def cross_entropy_mean(logits, targets):
    """src/Loss/CrossEntropy.php:36-85 restated: (mean loss, gradient)."""
    z = _f32(logits)
    t = np.ascontiguousarray(targets, np.int32)
    g = np.empty_like(z)
    loss = lib("oracle").oracle_cross_entropy_mean(z, t, g, z.shape[0], z.shape[1])
    return loss, g


# ---------------------------------------------------------------- whole step
class StepModel:
    """A model trained by the step driver cnn_step.c on the CPU C-ABI.

    spec: list of (kind, a, b, c) rows (1 conv3x3, 2 ReLU, 3 MaxPool2x2, 4 Linear).
    kind: "oracle" (restatement, strict) or "refstep" (reference library, its flags).
    """

    def __init__(self, spec, batch, in_shape, nthreads=1, kind="oracle"):
        self.L = lib(kind)
        s = np.ascontiguousarray(np.asarray(spec, np.int32).ravel())
        C_, H, W = in_shape
        self.h = self.L.zo_model_create(s, len(spec), batch, C_, H, W, nthreads)
        if not self.h:
            raise ValueError("bad model spec")
        self.n = self.L.zo_model_nparams(self.h)
        self.batch, self.spec = batch, spec

    def _view(self, ptr, n, dtype=np.float32):
        return np.ctypeslib.as_array(ptr, shape=(n,)).view(dtype)

    @property
    def params(self) -> np.ndarray:
        return self._view(self.L.zo_model_params(self.h), self.n)

    @property
    def grads(self) -> np.ndarray:
        return self._view(self.L.zo_model_grads(self.h), self.n)

    def output(self, layer: int, n: int) -> np.ndarray:
        return self._view(self.L.zo_model_output(self.h, layer), n).copy()

    def argmax(self, layer: int, n: int) -> np.ndarray:
        return np.ctypeslib.as_array(self.L.zo_model_argmax(self.h, layer), shape=(n,)).copy()

    def step(self, x, y, opt: int, lr: float) -> float:
        """opt 0: gradients only; 1: SGD; 2: Adam(0.9, 0.999, 1e-8).  Returns the loss sum."""
        loss = C.c_float(0.0)
        rc = self.L.zo_model_step(self.h, _f32(x).ravel(), _f32(y).ravel(), opt, lr, C.byref(loss))
        if rc:
            raise RuntimeError(f"zo_model_step failed ({rc})")
        return float(loss.value)

    def close(self):
        if self.h:
            self.L.zo_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
