"""Python handle on the fused training step of libzilla_b200.so (zilla_net_*)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import native
from .configs import ADAM, LmWorkload, Workload


class Net:
    """A Sequential trained by one C call per step (zilla_net_step)."""

    def __init__(self, workload: Workload, batch: int | None = None, precision: int | None = None):
        self.w = workload
        self.lib = native.load()
        self.batch = batch if batch is not None else workload.batch
        self.precision = workload.precision if precision is None else precision
        spec = np.ascontiguousarray(np.asarray(workload.layers, np.int32).ravel())
        c, h, wd = workload.in_shape
        self.id = self.lib.zilla_net_create(spec.ctypes.data_as(native.IP), len(workload.layers), self.batch,
                                            c, h, wd, self.precision)
        if self.id <= 0:
            raise RuntimeError(f"zilla_net_create failed: {native.last_error()}")
        self.nparams = int(self.lib.zilla_net_param_count(self.id))
        b1, b2, eps = workload.adam
        self._check(self.lib.zilla_net_set_optimizer(self.id, workload.optimizer, workload.lr, b1, b2, eps))
        self.params_id = self.lib.zilla_net_params_id(self.id)
        self.grads_id = self.lib.zilla_net_grads_id(self.id)

    def _check(self, rc: int) -> None:
        if rc != 0:
            raise RuntimeError(f"libzilla_b200 call failed ({rc}): {native.last_error()}")

    # ---- parameters
    def set_params(self, p: np.ndarray) -> None:
        p = np.ascontiguousarray(p, np.float32)
        assert p.size == self.nparams
        self._check(self.lib.zilla_buffer_upload(self.params_id, p.ctypes.data_as(native.FP), p.size))

    def params(self) -> np.ndarray:
        out = np.empty(self.nparams, np.float32)
        self._check(self.lib.zilla_buffer_download(self.params_id, out.ctypes.data_as(native.FP), self.nparams))
        return out

    def grads(self) -> np.ndarray:
        out = np.empty(self.nparams + 1, np.float32)
        self._check(self.lib.zilla_buffer_download(self.grads_id, out.ctypes.data_as(native.FP), self.nparams + 1))
        return out[: self.nparams]

    def argmax(self, layer: int, n: int) -> np.ndarray:
        i = self.lib.zilla_net_argmax_id(self.id, layer)
        if i <= 0:
            raise RuntimeError("no argmax for that layer")
        out = np.empty(n, np.float32)
        self._check(self.lib.zilla_buffer_download(i, out.ctypes.data_as(native.FP), n))
        return out.view(np.int32)

    # ---- steps
    def step_host(self, x: np.ndarray, y: np.ndarray, update: bool = True) -> float:
        x = np.ascontiguousarray(x, np.float32)
        y = np.ascontiguousarray(y, np.float32)
        loss = C.c_float(0.0)
        self._check(self.lib.zilla_net_step_host(self.id, x.ctypes.data_as(native.FP), y.ctypes.data_as(native.FP),
                                                 C.byref(loss), int(update)))
        return float(loss.value)

    def stage_host(self, x: np.ndarray, y: np.ndarray) -> None:
        """Enqueue the host->device copy of the next batch (zilla_net_stage_host);
        the arrays must stay alive and unchanged until its step_staged returns."""
        self._staged = getattr(self, "_staged", [])
        xa = x if (x.dtype == np.float32 and x.flags.c_contiguous) else np.ascontiguousarray(x, np.float32)
        ya = y if (y.dtype == np.float32 and y.flags.c_contiguous) else np.ascontiguousarray(y, np.float32)
        self._check(self.lib.zilla_net_stage_host(self.id, xa.ctypes.data_as(native.FP), ya.ctypes.data_as(native.FP)))
        self._staged.append((xa, ya))   # keep the host buffers alive until their step

    def step_staged(self, update: bool = True) -> float:
        """Step on the oldest staged batch (zilla_net_step_staged); returns the loss sum."""
        loss = C.c_float(0.0)
        self._check(self.lib.zilla_net_step_staged(self.id, C.byref(loss), int(update)))
        staged = getattr(self, "_staged", [])
        if staged:
            staged.pop(0)
        return float(loss.value)

    def step_staged_deferred(self, update: bool = True) -> float | None:
        """Step on the oldest staged batch without waiting for its loss
        (zilla_net_step_staged_deferred); returns the PREVIOUS deferred step's
        loss sum, or None on the first call."""
        loss, has = C.c_float(0.0), C.c_int(0)
        self._check(self.lib.zilla_net_step_staged_deferred(self.id, C.byref(loss), C.byref(has), int(update)))
        staged = getattr(self, "_staged", [])
        if staged:
            staged.pop(0)
        return float(loss.value) if has.value else None

    def loss_flush(self) -> float | None:
        """The last deferred step's loss sum (zilla_net_loss_flush), or None."""
        loss, has = C.c_float(0.0), C.c_int(0)
        self._check(self.lib.zilla_net_loss_flush(self.id, C.byref(loss), C.byref(has)))
        return float(loss.value) if has.value else None

    def forward(self, x: np.ndarray, y: np.ndarray | None = None) -> tuple[np.ndarray, float | None]:
        """Evaluation through zilla_net_forward: (logits [batch, classes], loss sum or None)."""
        lib, ids = self.lib, []

        def dev(a: np.ndarray) -> int:
            a = np.ascontiguousarray(a, np.float32)
            i = lib.zilla_buffer_alloc(a.size)
            if i <= 0:
                raise RuntimeError(f"zilla_buffer_alloc failed: {native.last_error()}")
            ids.append(i)
            self._check(lib.zilla_buffer_upload(i, a.ctypes.data_as(native.FP), a.size))
            return i

        try:
            xi = dev(x)
            yi = dev(y) if y is not None else 0
            li = dev(np.zeros(1, np.float32)) if y is not None else 0
            lo = dev(np.zeros(self.batch * self.w.classes, np.float32))
            self._check(lib.zilla_net_forward(self.id, xi, yi, lo, li))
            logits = np.empty(self.batch * self.w.classes, np.float32)
            self._check(lib.zilla_buffer_download(lo, logits.ctypes.data_as(native.FP), logits.size))
            loss = None
            if li:
                l1 = np.empty(1, np.float32)
                self._check(lib.zilla_buffer_download(li, l1.ctypes.data_as(native.FP), 1))
                loss = float(l1[0])
            return logits.reshape(self.batch, self.w.classes), loss
        finally:
            for i in ids:
                lib.zilla_buffer_free(i)

    def step_dev(self, x_id: int, y_id: int, loss_id: int, update: bool = True) -> None:
        self._check(self.lib.zilla_net_step(self.id, x_id, y_id, loss_id, int(update)))

    def set_graph(self, enable: bool = True) -> None:
        """Replay the step from a CUDA graph (zilla_net_set_graph)."""
        self._check(self.lib.zilla_net_set_graph(self.id, int(enable)))

    def profile(self, enable: bool = True) -> None:
        self._check(self.lib.zilla_net_profile(self.id, int(enable)))

    def profile_segment(self, segment: int) -> None:
        """Time only segment `segment` of each step (zilla_net_profile_segment)."""
        self._check(self.lib.zilla_net_profile_segment(self.id, segment))

    def timings(self) -> list[tuple[str, float]]:
        """(label, ms) of each kernel group of the last profiled step."""
        labels = C.create_string_buffer(8192)
        ms = np.zeros(256, np.float32)
        k = self.lib.zilla_net_timings(self.id, labels, 8192, ms.ctypes.data_as(native.FP), 256)
        if k < 0:
            raise RuntimeError(native.last_error())
        names = labels.value.decode().split("\n")[:k]
        return list(zip(names, ms[:k].tolist()))

    def device_status(self) -> None:
        """Raises if a kernel recorded an error (expired bounded wait, bad index)."""
        self._check(self.lib.zilla_net_device_status(self.id))

    def inspect(self) -> dict[str, np.ndarray]:
        """Intermediate tensors of the tensor-core engine (diagnostics), by name."""
        out, i = {}, 0
        while True:
            name = C.create_string_buffer(64)
            n = self.lib.zilla_net_inspect(self.id, i, name, 64, None, 0)
            if n <= 0:
                break
            buf = np.empty(n, np.float32)
            self._check(0 if self.lib.zilla_net_inspect(self.id, i, name, 64, buf.ctypes.data_as(native.FP), n) == n
                        else -3)
            out[name.value.decode()] = buf
            i += 1
        return out

    def dp_attach(self, rank: int, world: int, uid: bytes) -> None:
        self._check(self.lib.zilla_dp_attach(self.id, rank, world, uid))

    def close(self) -> None:
        if getattr(self, "id", 0) > 0:
            self.lib.zilla_net_destroy(self.id)
            self.id = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class LM(Net):
    """A Transformer language model trained by one C call per step
    (zilla_lm_create + zilla_net_step): x and y are the batch*seq token ids
    and next-token ids, as floats."""

    def __init__(self, workload: LmWorkload, batch: int | None = None, seq: int | None = None, precision: int = 0):
        self.w = workload
        self.lib = native.load()
        self.batch = batch if batch is not None else workload.batch
        self.seq = seq if seq is not None else workload.seq
        self.precision = precision
        w = workload
        self.id = self.lib.zilla_lm_create(w.vocab, w.dim, w.heads, w.layers, w.max_seq, w.ffn, self.batch,
                                           self.seq)
        if self.id <= 0:
            raise RuntimeError(f"zilla_lm_create failed: {native.last_error()}")
        self.nparams = int(self.lib.zilla_net_param_count(self.id))
        b1, b2, eps = w.adam
        self._check(self.lib.zilla_net_set_optimizer(self.id, w.optimizer, w.lr, b1, b2, eps))
        self.params_id = self.lib.zilla_net_params_id(self.id)
        self.grads_id = self.lib.zilla_net_grads_id(self.id)
        if precision:   # TF32 tensor-core GEMMs for the blocks' Linear layers
            self._check(self.lib.zilla_lm_set_precision(self.id, precision))

    def forward_cached(self, tokens) -> np.ndarray:
        """TransformerLM::forwardWithCache: logits [len(tokens), vocab] for the
        tokens at the next cache positions; the cache grows by len(tokens)."""
        t = np.ascontiguousarray(tokens, np.float32).ravel()
        out = np.empty((t.size, self.w.vocab), np.float32)
        self._check(self.lib.zilla_lm_forward_cached(self.id, t.ctypes.data_as(native.FP), t.size,
                                                     out.ctypes.data_as(native.FP)))
        return out

    def cache_reset(self) -> None:
        self._check(self.lib.zilla_lm_cache_reset(self.id))

    def cache_length(self) -> int:
        n = int(self.lib.zilla_lm_cache_length(self.id))
        if n < 0:
            raise RuntimeError(native.last_error())
        return n


def dp_unique_id() -> bytes:
    lib = native.load()
    buf = C.create_string_buffer(128)
    if lib.zilla_dp_unique_id(buf) != 0:
        raise RuntimeError(native.last_error())
    return buf.raw


def is_adam(w: Workload) -> bool:
    return w.optimizer == ADAM
