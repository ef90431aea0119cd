"""Loads libzilla_b200.so and declares the C-ABI of include/zilla_b200.h for ctypes.

The library is the product: there is no fallback.  If it is missing the
loader raises, telling the caller to build it (``python -m zillaphp_b200.build``).
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libzilla_b200.so")

I, F, VP, UL = C.c_int, C.c_float, C.c_void_p, C.c_ulong
FP = C.POINTER(C.c_float)
IP = C.POINTER(C.c_int)

# name -> (restype, argtypes); every function of include/zilla_b200.h
SIGNATURES: dict[str, tuple] = {
    # host-pointer helpers
    "matmul_f32": (None, [FP, FP, FP, I, I, I]),
    "relu_f32_cuda": (None, [FP, FP, I]),
    "add_f32_cuda": (None, [FP, FP, FP, I]),
    "sub_f32_cuda": (None, [FP, FP, FP, I]),
    "mul_f32_cuda": (None, [FP, FP, FP, I]),
    "div_f32_cuda": (None, [FP, FP, FP, I]),
    "hann_window_cuda": (None, [FP, I]),
    "stft_magnitude_cuda": (None, [FP, I, FP, I, I, FP, IP, IP]),
    # registry
    "zilla_buffer_alloc": (I, [UL]),
    "zilla_buffer_free": (None, [I]),
    "zilla_buffer_upload": (I, [I, FP, UL]),
    "zilla_buffer_download": (I, [I, FP, UL]),
    "zilla_sync": (None, []),
    "zilla_buffer_ptr": (VP, [I]),
    # device ops
    "matmul_dev": (I, [I, I, I, I, I, I]),
    "add_dev": (I, [I, I, I, I]),
    "sub_dev": (I, [I, I, I, I]),
    "mul_dev": (I, [I, I, I, I]),
    "div_dev": (I, [I, I, I, I]),
    "relu_dev": (I, [I, I, I]),
    # training ops
    "add_bias_dev": (I, [I, I, I, I]),
    "relu_fwd_dev": (I, [I, I, I, I]),
    "relu_bwd_dev": (I, [I, I, I, I]),
    "softmax_ce_dev": (I, [I, I, I, I, I, I]),
    "bias_grad_dev": (I, [I, I, I, I]),
    "sgd_update_dev": (I, [I, I, F, I]),
    "zero_dev": (I, [I, I]),
    "matmul_tn_dev": (I, [I, I, I, I, I, I]),
    "matmul_nt_dev": (I, [I, I, I, I, I, I]),
    "copy_dev": (I, [I, I, I]),
    # conv / pool
    "conv2d_fwd_dev": (I, [I] * 14),
    "conv2d_bwd_dev": (I, [I] * 16),
    "maxpool2d_fwd_dev": (I, [I] * 11),
    "maxpool2d_bwd_dev": (I, [I] * 6),
    "conv2d_batched_fwd_dev": (I, [I] * 15),
    "conv2d_batched_bwd_dev": (I, [I] * 17),
    "maxpool2d_batched_fwd_dev": (I, [I] * 12),
    "maxpool2d_batched_bwd_dev": (I, [I] * 7),
    # attention
    "softmax_rows_fwd_dev": (I, [I, I, I, I]),
    "softmax_rows_bwd_dev": (I, [I, I, I, I, I]),
    "causal_mask_dev": (I, [I, I, I, F]),
    "scale_dev": (I, [I, F, I]),
    "causal_softmax_dev": (I, [I, I, I, F]),
    # additive
    "zilla_last_error": (C.c_char_p, []),
    "zilla_last_status": (I, []),
    "zilla_set_stream": (I, [VP]),
    "zilla_launch_count": (C.c_ulonglong, []),
    "zilla_check_device": (I, []),
    "adam_update_dev": (I, [I, I, I, I, F, F, F, F, I, I]),
    "softmax_ce_clamped_dev": (I, [I, I, I, I, I, I]),
    "softmax_ce_noalloc": (I, [VP, VP, VP, VP, I, I, VP]),
    "zilla_net_create": (I, [IP, I, I, I, I, I, I]),
    "zilla_net_destroy": (I, [I]),
    "zilla_net_param_count": (C.c_long, [I]),
    "zilla_net_params_id": (I, [I]),
    "zilla_net_grads_id": (I, [I]),
    "zilla_net_argmax_id": (I, [I, I]),
    "zilla_net_set_optimizer": (I, [I, I, F, F, F, F]),
    "zilla_net_step": (I, [I, I, I, I, I]),
    "zilla_net_step_host": (I, [I, FP, FP, FP, I]),
    "zilla_net_stage_host": (I, [I, FP, FP]),
    "zilla_net_forward": (I, [I, I, I, I, I]),
    "zilla_net_set_graph": (I, [I, I]),
    "zilla_net_save": (I, [I, C.c_char_p, I]),
    "zilla_net_load": (I, [I, C.c_char_p]),
    "zilla_net_step_staged": (I, [I, FP, I]),
    "zilla_net_step_staged_deferred": (I, [I, FP, IP, I]),
    "zilla_net_loss_flush": (I, [I, FP, IP]),
    "zilla_net_profile": (I, [I, I]),
    "zilla_net_profile_segment": (I, [I, I]),
    "zilla_net_timings": (I, [I, C.c_char_p, I, FP, I]),
    "zilla_net_inspect": (I, [I, I, C.c_char_p, I, FP, UL]),
    "zilla_net_device_status": (I, [I]),
    "zilla_lm_create": (I, [I] * 8),
    "zilla_lm_forward_cached": (I, [I, FP, I, FP]),
    "zilla_lm_cache_reset": (I, [I]),
    "zilla_lm_set_precision": (I, [I, I]),
    "zilla_lm_cache_length": (I, [I]),
    "zilla_dp_unique_id": (I, [C.c_char_p]),
    "zilla_dp_attach": (I, [I, I, I, C.c_char_p]),
    "zilla_dp_detach": (I, [I]),
}

_lib: C.CDLL | None = None


def load() -> C.CDLL:
    """Returns the loaded library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m zillaphp_b200.build` "
            "(there is no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    return load().zilla_last_error().decode(errors="replace")
