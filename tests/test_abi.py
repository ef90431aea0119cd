"""The C-ABI library loads and exports every symbol it declares (CPU only).

No compute is issued here: the calls below fail on host-side argument
checks before any device work, which is itself the error contract
(0 ok, -1 bad handle / capacity, -2 bad argument).
"""
import ctypes as C
import os
import re

import numpy as np
import pytest

from zillaphp_b200 import configs, native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# The FFI::cdef block of src/Hardware/CUDA/CudaBackend.php:51-95.
PHP_CDEF = """
matmul_f32 relu_f32_cuda add_f32_cuda sub_f32_cuda mul_f32_cuda div_f32_cuda hann_window_cuda
stft_magnitude_cuda zilla_buffer_alloc zilla_buffer_free zilla_buffer_upload zilla_buffer_download
zilla_sync matmul_dev add_dev sub_dev mul_dev div_dev relu_dev add_bias_dev relu_fwd_dev relu_bwd_dev
softmax_ce_dev bias_grad_dev sgd_update_dev zero_dev matmul_tn_dev matmul_nt_dev copy_dev
conv2d_fwd_dev conv2d_bwd_dev maxpool2d_fwd_dev maxpool2d_bwd_dev conv2d_batched_fwd_dev
conv2d_batched_bwd_dev maxpool2d_batched_fwd_dev maxpool2d_batched_bwd_dev softmax_rows_fwd_dev
softmax_rows_bwd_dev causal_mask_dev scale_dev causal_softmax_dev
""".split()


def header_functions():
    text = open(os.path.join(ROOT, "include", "zilla_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b([a-z_][a-z0-9_]*)\s*\(", text)) - {"if", "sizeof"})


@pytest.fixture(scope="module")
def lib():
    return native.load()


def test_header_declares_reference_cdef():
    decl = set(header_functions())
    missing = [f for f in PHP_CDEF if f not in decl]
    assert not missing, missing


def test_library_exports_every_declared_symbol(lib):
    raw = C.CDLL(native.LIB_PATH)
    missing = [f for f in header_functions() if not hasattr(raw, f)]
    assert not missing, missing
    assert set(header_functions()) <= set(native.SIGNATURES)


def test_host_side_errors(lib):
    assert lib.zilla_buffer_alloc(0) == -1
    assert "zero size" in native.last_error()
    assert lib.zilla_buffer_ptr(0) is None
    assert lib.zilla_buffer_ptr(8191) is None
    assert lib.zilla_buffer_ptr(9000) is None
    lib.zilla_buffer_free(-3)          # idempotent no-op
    lib.zilla_buffer_free(77)
    for rc in (lib.relu_dev(77, 78, 10), lib.matmul_dev(1, 2, 3, 4, 5, 6),
               lib.softmax_ce_dev(1, 2, 3, 4, 8, 10), lib.softmax_ce_clamped_dev(1, 2, 3, 4, 8, 10),
               lib.conv2d_batched_fwd_dev(*([5] * 15)),
               lib.maxpool2d_batched_bwd_dev(1, 2, 3, 4, 5, 6, 7), lib.adam_update_dev(1, 2, 3, 4, 1e-3, .9, .999, 1e-8, 1, 8)):
        assert rc == -1
    buf = np.zeros(4, np.float32)
    assert lib.zilla_buffer_upload(5, buf.ctypes.data_as(native.FP), 4) == -1
    assert lib.zilla_buffer_download(5, buf.ctypes.data_as(native.FP), 4) == -1


def test_net_spec_validation(lib):
    def create(layers, batch=4, shape=(1, 28, 28), precision=0):
        spec = np.ascontiguousarray(np.asarray(layers, np.int32).ravel())
        return lib.zilla_net_create(spec.ctypes.data_as(native.IP), len(layers), batch, *shape, precision)
    assert create([(1, 3, 8, 1)]) == -2                         # wrong input channels
    assert create([(4, 100, 10, 0)]) == -2                      # Linear size mismatch
    assert create([(9, 0, 0, 0)]) == -2                        # unknown layer kind
    assert create([(4, 784, 10, 0)], precision=5) == -2        # bad precision
    assert create([(4, 784, 10, 0)], batch=0) == -2
    assert lib.zilla_net_step(12345, 1, 2, 3, 1) == -1          # unknown net
    assert lib.zilla_net_destroy(12345) == -1


def test_lm_create_validation(lib):
    ok = (65, 128, 4, 2, 128, 512, 64, 128)
    def create(**kw):
        args = dict(zip(("vocab", "dim", "heads", "layers", "max_seq", "ffn", "batch", "seq"), ok))
        args.update(kw)
        return lib.zilla_lm_create(*args.values())
    assert create(heads=8) == -2                # head dimension 16: only 32 is built
    assert create(seq=129) == -2                # longer than the position table
    assert create(max_seq=512, seq=200) == -2   # attention backward tile beyond shared memory
    assert create(vocab=0) == -2
    assert create(batch=0) == -2


def test_workload_param_counts():
    assert configs.param_count(configs.CNN_LARGE) == 1_701_130
    assert configs.param_count(configs.AUDIO_CNN) == 97_036
    assert configs.param_count(configs.MLP) == 101_770
    assert configs.param_count(configs.CNN_SMALL) == 13_610
    assert configs.lm_param_count(configs.TRANSFORMER_LM) == 429_889
    assert abs(configs.flops_per_sample(configs.CNN_LARGE) * 8192 / 1e9 - 1507.0) < 1.0
