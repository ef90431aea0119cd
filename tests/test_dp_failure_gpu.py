"""Failure detection of the data-parallel step over peer memory (two GPUs;
skipped with fewer).  The failure is made on the host: after a first step
together, rank 1 stays alive but does not take the second step (no kernel of
it in flight).  Rank 0's update kernel then waits for rank 1's "gradients
final" flag until its bounded wait expires, records 0x50450001 in the device
error word and returns, and its final wait for rank 1's slice expires the same
way; the host sees the error through zilla_net_device_status, and rank 0's GPU
context stays usable (a buffer round trip afterwards).  NVLS is off and only
plain peer loads/stores are used; no GPU fault, trap or hang is involved.
"""
import os
import sys
import time

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _rank(rank, uid_q, out_q, go_q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path[:0] = [ROOT]
    import torch
    torch.cuda.set_device(rank)
    from zillaphp_b200 import configs, native, synthetic
    from zillaphp_b200.net import Net, dp_unique_id
    try:
        w = configs.CNN_LARGE
        net = Net(w, batch=64, precision=1)
        net.set_params(synthetic.init_params(w, seed=4))
        if rank == 0:
            uid = dp_unique_id()
            uid_q.put(uid)
        else:
            uid = uid_q.get(timeout=60)
        net.dp_attach(rank, 2, uid)
        x, y = synthetic.batch(w, 128, seed=4, step=0)
        net.step_host(x[rank * 64:(rank + 1) * 64], y[rank * 64:(rank + 1) * 64])
        net.device_status()   # the first step together is clean
        if rank == 1:
            go_q.get(timeout=120)   # alive, between steps, until rank 0 has seen the failure
            out_q.put((rank, "idle", None))
        else:
            x, y = synthetic.batch(w, 128, seed=4, step=1)
            t0 = time.time()
            net.step_host(x[:64], y[:64])
            err = None
            try:
                net.device_status()
            except RuntimeError as e:
                err = str(e)
            waited = time.time() - t0
            # the context still works after the expired waits
            lib = native.load()
            buf = lib.zilla_buffer_alloc(16)
            a = np.arange(16, dtype=np.float32)
            back = np.empty(16, np.float32)
            ok = (buf > 0 and lib.zilla_buffer_upload(buf, a.ctypes.data_as(native.FP), 16) == 0 and
                  lib.zilla_buffer_download(buf, back.ctypes.data_as(native.FP), 16) == 0 and
                  np.array_equal(a, back))
            lib.zilla_buffer_free(buf)
            go_q.put(True)
            out_q.put((rank, (err, waited, ok), None))
        net.close()
    except Exception as e:  # noqa: BLE001
        try:
            go_q.put(True)
        except Exception:
            pass
        out_q.put((rank, None, repr(e)))


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.timeout(300)
def test_peer_step_reports_a_rank_that_does_not_step():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    uid_q, out_q, go_q = ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, uid_q, out_q, go_q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, val, err = out_q.get(timeout=240)
            assert err is None, f"rank {rank}: {err}"
            res[rank] = val
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    err, waited, ok = res[0]
    assert err is not None and "0x50450001" in err, err
    assert 1.5 < waited < 60, waited
    assert ok, "rank 0's context was not usable after the expired waits"
