"""Host-side mirror of ZillaPHP's CudaBackend over libzilla_b200.so.

Same method names, argument order and error behaviour as
src/Hardware/CUDA/CudaBackend.php:402-779: every ``*Dev`` call forwards to the
C function of the same name and raises ``RuntimeError("<fn> failed.")`` when it
returns non-zero; ``bufferAlloc`` raises on a negative handle, ``bufferFree`` is
a no-op for invalid handles.  Host arrays are numpy float32 arrays (PHP float
arrays in the reference).  This is the interface the parity tests drive; a
PHP host binds the same C functions through FFI::cdef.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import native


class ZillaError(RuntimeError):
    pass


def _fp(a: np.ndarray):
    return a.ctypes.data_as(native.FP)


class B200Backend:
    """The B200 counterpart of ``ZillaPHP\\Hardware\\CUDA\\CudaBackend``."""

    def __init__(self):
        self.ffi = native.load()

    def name(self) -> str:
        return "cuda"

    def isCuda(self) -> bool:  # noqa: N802 (reference method name)
        return True

    # ------------------------------------------------------------ helpers
    def _check(self, rc: int, fn: str) -> None:
        if rc != 0:
            raise ZillaError(f"{fn} failed. ({native.last_error()})")

    # ------------------------------------------------------------ registry
    def bufferAlloc(self, nFloats: int) -> int:  # noqa: N802,N803
        if nFloats < 1:
            raise ValueError("nFloats must be >= 1.")
        i = self.ffi.zilla_buffer_alloc(nFloats)
        if i < 0:
            raise ZillaError(f"zilla_buffer_alloc({nFloats}) failed — GPU out of memory?")
        return i

    def bufferFree(self, id: int) -> None:  # noqa: A002,N802
        if id > 0:
            self.ffi.zilla_buffer_free(id)

    def bufferUpload(self, id: int, host) -> None:  # noqa: A002,N802
        if id < 1:
            raise ValueError(f"Invalid buffer id: {id}")
        a = np.ascontiguousarray(host, dtype=np.float32).ravel()
        if self.ffi.zilla_buffer_upload(id, _fp(a), a.size) != 0:
            raise ZillaError(f"zilla_buffer_upload failed for id {id} ({a.size} floats).")

    def bufferUploadInt(self, id: int, host) -> None:  # noqa: A002,N802
        """Uploads int32 data (argmax) bit-for-bit into a float buffer."""
        a = np.ascontiguousarray(host, dtype=np.int32).ravel().view(np.float32)
        self.bufferUpload(id, a)

    def bufferDownload(self, id: int, nFloats: int) -> np.ndarray:  # noqa: A002,N802,N803
        out = np.empty(nFloats, np.float32)
        if self.ffi.zilla_buffer_download(id, _fp(out), nFloats) != 0:
            raise ZillaError(f"zilla_buffer_download failed for id {id}.")
        return out

    def bufferDownloadInt(self, id: int, n: int) -> np.ndarray:  # noqa: A002,N802
        return self.bufferDownload(id, n).view(np.int32)

    def sync(self) -> None:
        self.ffi.zilla_sync()

    # ------------------------------------------------------------ device ops
    def matmulDev(self, aId, bId, cId, m, k, n):  # noqa: N802,N803
        self._check(self.ffi.matmul_dev(aId, bId, cId, m, k, n), f"matmul_dev({aId}, {bId}, {cId}, {m}, {k}, {n})")

    def addDev(self, aId, bId, cId, n):  # noqa: N802,N803
        self._check(self.ffi.add_dev(aId, bId, cId, n), "add_dev")

    def subDev(self, aId, bId, cId, n):  # noqa: N802,N803
        self._check(self.ffi.sub_dev(aId, bId, cId, n), "sub_dev")

    def mulDev(self, aId, bId, cId, n):  # noqa: N802,N803
        self._check(self.ffi.mul_dev(aId, bId, cId, n), "mul_dev")

    def divDev(self, aId, bId, cId, n):  # noqa: N802,N803
        self._check(self.ffi.div_dev(aId, bId, cId, n), "div_dev")

    def reluDev(self, xId, yId, n):  # noqa: N802,N803
        self._check(self.ffi.relu_dev(xId, yId, n), "relu_dev")

    # ------------------------------------------------------------ training ops
    def addBiasDev(self, xId, bId, B, C_):  # noqa: N802,N803
        self._check(self.ffi.add_bias_dev(xId, bId, B, C_), "add_bias_dev")

    def reluFwdDev(self, xId, yId, maskId, n):  # noqa: N802,N803
        self._check(self.ffi.relu_fwd_dev(xId, yId, maskId, n), "relu_fwd_dev")

    def reluBwdDev(self, dyId, maskId, dxId, n):  # noqa: N802,N803
        self._check(self.ffi.relu_bwd_dev(dyId, maskId, dxId, n), "relu_bwd_dev")

    def softmaxCeDev(self, logitsId, targetsId, dlogitsId, lossId, B, C_):  # noqa: N802,N803
        self._check(self.ffi.softmax_ce_dev(logitsId, targetsId, dlogitsId, lossId, B, C_), "softmax_ce_dev")

    def softmaxCeClampedDev(self, logitsId, targetsId, dlogitsId, lossId, B, C_):  # noqa: N802,N803
        self._check(self.ffi.softmax_ce_clamped_dev(logitsId, targetsId, dlogitsId, lossId, B, C_),
                    "softmax_ce_clamped_dev")

    def biasGradDev(self, dyId, dbId, B, C_):  # noqa: N802,N803
        self._check(self.ffi.bias_grad_dev(dyId, dbId, B, C_), "bias_grad_dev")

    def sgdUpdateDev(self, wId, dwId, lr, n):  # noqa: N802,N803
        self._check(self.ffi.sgd_update_dev(wId, dwId, lr, n), "sgd_update_dev")

    def adamUpdateDev(self, wId, gId, mId, vId, lr, beta1, beta2, eps, t, n):  # noqa: N802,N803
        self._check(self.ffi.adam_update_dev(wId, gId, mId, vId, lr, beta1, beta2, eps, t, n), "adam_update_dev")

    def zeroDev(self, id, n):  # noqa: A002,N802
        self._check(self.ffi.zero_dev(id, n), "zero_dev")

    def matmulTnDev(self, aId, bId, cId, M, K, N):  # noqa: N802,N803
        self._check(self.ffi.matmul_tn_dev(aId, bId, cId, M, K, N), "matmul_tn_dev")

    def matmulNtDev(self, aId, bId, cId, M, K, N):  # noqa: N802,N803
        self._check(self.ffi.matmul_nt_dev(aId, bId, cId, M, K, N), "matmul_nt_dev")

    def copyDev(self, srcId, dstId, n):  # noqa: N802,N803
        self._check(self.ffi.copy_dev(srcId, dstId, n), "copy_dev")

    # ------------------------------------------------------------ conv / pool
    def conv2dFwdDev(self, inputId, weightId, biasId, outputId, C_, H, W, outC, outH, outW, kH, kW, stride, padding):  # noqa: N802,N803,E501
        self._check(self.ffi.conv2d_fwd_dev(inputId, weightId, biasId, outputId, C_, H, W, outC, outH, outW,
                                            kH, kW, stride, padding), "conv2d_fwd_dev")

    def conv2dBwdDev(self, inputId, weightId, gradOutId, gradInputId, gradWeightId, gradBiasId, C_, H, W,  # noqa: N802,N803
                     outC, outH, outW, kH, kW, stride, padding):  # noqa: N803
        self._check(self.ffi.conv2d_bwd_dev(inputId, weightId, gradOutId, gradInputId, gradWeightId, gradBiasId,
                                            C_, H, W, outC, outH, outW, kH, kW, stride, padding), "conv2d_bwd_dev")

    def maxPool2dFwdDev(self, inputId, outputId, argmaxId, C_, H, W, outH, outW, kH, kW, stride):  # noqa: N802,N803
        self._check(self.ffi.maxpool2d_fwd_dev(inputId, outputId, argmaxId, C_, H, W, outH, outW, kH, kW, stride),
                    "maxpool2d_fwd_dev")

    def maxPool2dBwdDev(self, gradOutId, argmaxId, gradInputId, C_, outH, outW):  # noqa: N802,N803
        self._check(self.ffi.maxpool2d_bwd_dev(gradOutId, argmaxId, gradInputId, C_, outH, outW), "maxpool2d_bwd_dev")

    def conv2dBatchedFwdDev(self, inputId, weightId, biasId, outputId, B, C_, H, W, outC, outH, outW,  # noqa: N802,N803
                            kH, kW, stride, padding):  # noqa: N803
        self._check(self.ffi.conv2d_batched_fwd_dev(inputId, weightId, biasId, outputId, B, C_, H, W, outC, outH,
                                                    outW, kH, kW, stride, padding), "conv2d_batched_fwd_dev")

    def conv2dBatchedBwdDev(self, inputId, weightId, gradOutId, gradInputId, gradWeightId, gradBiasId, B, C_,  # noqa: N802,N803,E501
                            H, W, outC, outH, outW, kH, kW, stride, padding):  # noqa: N803
        self._check(self.ffi.conv2d_batched_bwd_dev(inputId, weightId, gradOutId, gradInputId, gradWeightId,
                                                    gradBiasId, B, C_, H, W, outC, outH, outW, kH, kW, stride,
                                                    padding), "conv2d_batched_bwd_dev")

    def maxPool2dBatchedFwdDev(self, inputId, outputId, argmaxId, B, C_, H, W, outH, outW, kH, kW, stride):  # noqa: N802,N803,E501
        self._check(self.ffi.maxpool2d_batched_fwd_dev(inputId, outputId, argmaxId, B, C_, H, W, outH, outW, kH, kW,
                                                       stride), "maxpool2d_batched_fwd_dev")

    def maxPool2dBatchedBwdDev(self, gradOutId, argmaxId, gradInputId, B, C_, outH, outW):  # noqa: N802,N803
        self._check(self.ffi.maxpool2d_batched_bwd_dev(gradOutId, argmaxId, gradInputId, B, C_, outH, outW),
                    "maxpool2d_batched_bwd_dev")

    # ------------------------------------------------------------ attention
    def softmaxRowsFwdDev(self, xId, yId, N, M):  # noqa: N802,N803
        self._check(self.ffi.softmax_rows_fwd_dev(xId, yId, N, M), "softmax_rows_fwd_dev")

    def softmaxRowsBwdDev(self, pId, dpId, dsId, N, M):  # noqa: N802,N803
        self._check(self.ffi.softmax_rows_bwd_dev(pId, dpId, dsId, N, M), "softmax_rows_bwd_dev")

    def causalMaskDev(self, xId, N, M, maskValue=-1e9):  # noqa: N802,N803
        self._check(self.ffi.causal_mask_dev(xId, N, M, maskValue), "causal_mask_dev")

    def scaleDev(self, xId, scale, n):  # noqa: N802,N803
        self._check(self.ffi.scale_dev(xId, scale, n), "scale_dev")

    def causalSoftmaxDev(self, xId, N, M, maskValue=-1e9):  # noqa: N802,N803
        self._check(self.ffi.causal_softmax_dev(xId, N, M, maskValue), "causal_softmax_dev")

    # ------------------------------------------------------------ host-pointer helpers
    def matmul(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        out = np.empty((a.shape[0], b.shape[1]), np.float32)
        self.ffi.matmul_f32(_fp(a), _fp(b), _fp(out), a.shape[0], a.shape[1], b.shape[1])
        return out

    def elementwise(self, op: str, a: np.ndarray, b: np.ndarray | None = None) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32).ravel()
        out = np.empty_like(a)
        if op == "relu":
            self.ffi.relu_f32_cuda(_fp(a), _fp(out), a.size)
        else:
            b = np.ascontiguousarray(b, np.float32).ravel()
            getattr(self.ffi, f"{op}_f32_cuda")(_fp(a), _fp(b), _fp(out), a.size)
        return out

    def hannWindow(self, n: int) -> np.ndarray:  # noqa: N802
        out = np.empty(n, np.float32)
        self.ffi.hann_window_cuda(_fp(out), n)
        return out

    def stftMagnitude(self, x: np.ndarray, fftSize: int, hopSize: int) -> np.ndarray:  # noqa: N802,N803
        x = np.ascontiguousarray(x, np.float32)
        nb, nf = C.c_int(0), C.c_int(0)
        n_frames_max = max(1, 1 + (x.size - fftSize) // hopSize) if x.size >= fftSize else 1
        out = np.zeros((fftSize // 2 + 1) * n_frames_max, np.float32)
        self.ffi.stft_magnitude_cuda(_fp(x), x.size, None, fftSize, hopSize, _fp(out), C.byref(nb), C.byref(nf))
        return out[: nb.value * nf.value].reshape(nb.value, nf.value)
