"""softmax_ce_noalloc: the allocation-free softmax cross-entropy (GPU).

Some callers cannot let a library allocate device memory: code that runs under
a caller-owned memory pool or budget, or a host that only hands over device
pointers it already owns.  softmax_ce_noalloc serves them with the per-row
scratch in a static device array instead of a cudaMalloc'd buffer.  This test
calls it through the C-ABI on raw device pointers, twice in a row with
different shapes, and checks each result against softmax_ce_dev (the existing
entry point) with the tolerance the other softmax-CE tests use (1e-5).  It
passes alone in a fresh process and after the rest of the suite.
"""
import ctypes as C

import numpy as np
import pytest

import npref
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
    # allocation-free entry point (raw device pointers, legacy default stream)
    ptr = lib.zilla_buffer_ptr
    rc = lib.softmax_ce_noalloc(ptr(iz), ptr(it), ptr(idz2), ptr(il2), B, Cn, None)
    assert rc == 0, native.last_error()
    be.sync()
    ref_dz, ref_l = be.bufferDownload(idz, B * Cn), float(be.bufferDownload(il, 1)[0])
    got_dz, got_l = be.bufferDownload(idz2, B * Cn), float(be.bufferDownload(il2, 1)[0])
    for i in ids:
        be.bufferFree(i)
    return ref_dz, ref_l, got_dz, got_l


def test_noalloc_matches_softmax_ce_dev_twice():
    be = B200Backend()
    lib = native.load()
    for B, Cn, seed in ((64, 10, 1), (8192, 65, 2)):       # two calls in a row, different sizes
        ref_dz, ref_l, got_dz, got_l = _case(be, lib, B, Cn, seed)
        assert npref.normwise(got_dz, ref_dz) < 1e-5
        assert abs(got_l - ref_l) / abs(ref_l) < 1e-5


def test_noalloc_rejects_batches_beyond_its_scratch():
    lib = native.load()
    dummy = C.c_void_p(16)   # never dereferenced: the size check comes first
    assert lib.softmax_ce_noalloc(dummy, dummy, dummy, dummy, 65537, 10, None) == -2
    assert "exceeds" in native.last_error()
