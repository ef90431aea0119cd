"""softmax_ce_noalloc: the allocation-free softmax cross-entropy (GPU).

Some callers cannot let a library allocate device memory: code that runs under
a caller-owned memory pool or budget, or a host that only hands over device
pointers it already owns.  softmax_ce_noalloc serves them with the per-row
scratch in a static device array instead of a cudaMalloc'd buffer.  These
tests call it through the C-ABI on raw device pointers:
  - twice in a row with different shapes, each result checked against
    softmax_ce_dev (the existing entry point) and against the oracle's
    softmax_ce_dev, with the tolerance the other softmax-CE tests use (1e-5);
  - on logits that a library op (matmul_dev) has just produced, with no host
    synchronisation in between and a NULL stream (the library's own stream),
    so the call must be ordered after the op that wrote its input;
  - with a batch beyond its scratch, which it rejects.
The file is collected last; it passes alone in a fresh process and after the
rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest

import npref
import oracle
from zillaphp_b200 import native
from zillaphp_b200.backend import B200Backend

pytestmark = pytest.mark.gpu


def _case(be, lib, B, Cn, seed):
    g = np.random.default_rng(seed)
    z = (g.standard_normal((B, Cn)) * 3).astype(np.float32)
    t = g.integers(0, Cn, B).astype(np.float32)
    ids = [be.bufferAlloc(B * Cn), be.bufferAlloc(B), be.bufferAlloc(B * Cn), be.bufferAlloc(1),
           be.bufferAlloc(B * Cn), be.bufferAlloc(1)]
    iz, it, idz, il, idz2, il2 = ids
    be.bufferUpload(iz, z)
    be.bufferUpload(it, t)
    be.bufferUpload(il, [0.0])
    be.bufferUpload(il2, [0.0])
    # existing entry point (registry handles, library scratch)
    be.softmaxCeDev(iz, it, idz, il, B, Cn)
    # allocation-free entry point (raw device pointers, the library's stream)
    ptr = lib.zilla_buffer_ptr
    rc = lib.softmax_ce_noalloc(ptr(iz), ptr(it), ptr(idz2), ptr(il2), B, Cn, None)
    assert rc == 0, native.last_error()
    be.sync()
    ref_dz, ref_l = be.bufferDownload(idz, B * Cn), float(be.bufferDownload(il, 1)[0])
    got_dz, got_l = be.bufferDownload(idz2, B * Cn), float(be.bufferDownload(il2, 1)[0])
    for i in ids:
        be.bufferFree(i)
    return z, t, ref_dz, ref_l, got_dz, got_l


def test_noalloc_matches_softmax_ce_dev_twice():
    be = B200Backend()
    lib = native.load()
    for B, Cn, seed in ((64, 10, 1), (8192, 65, 2)):       # two calls in a row, different sizes
        z, t, ref_dz, ref_l, got_dz, got_l = _case(be, lib, B, Cn, seed)
        assert npref.normwise(got_dz, ref_dz) < 1e-5
        assert abs(got_l - ref_l) / abs(ref_l) < 1e-5
        o_dz, o_l = oracle.softmax_ce_dev(z, t)            # the oracle directly
        assert npref.normwise(got_dz, o_dz.ravel()) < 1e-5
        assert abs(got_l - o_l) / abs(o_l) < 1e-5


def test_noalloc_ordered_after_library_ops():
    """Logits from matmul_dev, then softmax_ce_noalloc(..., NULL) with no host
    synchronisation between them: the NULL stream is the library's stream."""
    be = B200Backend()
    lib = native.load()
    g = np.random.default_rng(7)
    B, K, Cn = 4096, 256, 10
    x = g.standard_normal((B, K)).astype(np.float32)
    w = (g.standard_normal((K, Cn)) * 0.2).astype(np.float32)
    t = g.integers(0, Cn, B).astype(np.float32)
    ix, iw, iz, it, idz, il = (be.bufferAlloc(B * K), be.bufferAlloc(K * Cn), be.bufferAlloc(B * Cn),
                               be.bufferAlloc(B), be.bufferAlloc(B * Cn), be.bufferAlloc(1))
    be.bufferUpload(ix, x)
    be.bufferUpload(iw, w)
    be.bufferUpload(it, t)
    be.bufferUpload(il, [0.0])
    for _ in range(2):   # the second round overwrites the logits the first one consumed
        be.zeroDev(iz, B * Cn)
        be.zeroDev(il, 1)
        be.matmulDev(ix, iw, iz, B, K, Cn)
        ptr = lib.zilla_buffer_ptr
        assert lib.softmax_ce_noalloc(ptr(iz), ptr(it), ptr(idz), ptr(il), B, Cn, None) == 0, native.last_error()
        got_dz, got_l = be.bufferDownload(idz, B * Cn), float(be.bufferDownload(il, 1)[0])
        z = be.bufferDownload(iz, B * Cn).reshape(B, Cn)
        assert npref.normwise(z, oracle.matmul_dev(x, w)) < 1e-5
        o_dz, o_l = oracle.softmax_ce_dev(z, t)
        assert npref.normwise(got_dz, o_dz.ravel()) < 1e-5
        assert abs(got_l - o_l) / abs(o_l) < 1e-5
    for i in (ix, iw, iz, it, idz, il):
        be.bufferFree(i)


def test_noalloc_rejects_batches_beyond_its_scratch():
    lib = native.load()
    dummy = C.c_void_p(16)   # never dereferenced: the size check comes first
    assert lib.softmax_ce_noalloc(dummy, dummy, dummy, dummy, 65537, 10, None) == -2
    assert "exceeds" in native.last_error()
