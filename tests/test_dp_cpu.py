"""Data-parallel host logic on CPU ranks (gloo, world size 2).

What the GPU runner does per step, with the oracle standing in for the GPU
step (the device path itself is covered by the GPU tests):
  * each rank trains its contiguous 1/N shard of the global batch;
  * the flat gradient buffer with the loss sum in its last slot is summed
    over ranks (NCCL all-reduce on the GPUs, gloo here);
  * every rank scales by 1/N and applies the identical optimizer update.
The result must equal the single-process step on the whole batch, and the
128-byte communicator id must reach every rank unchanged (bench.py sends it
with broadcast_object_list).
"""
import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rank_main(rank, world, port, q):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
    import torch
    import torch.distributed as dist
    import oracle
    from zillaphp_b200 import configs, synthetic
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = configs.CNN_SMALL
        gb = 16
        b = gb // world
        x, y = synthetic.batch(w, gb, seed=9)
        p0 = synthetic.init_params(w, seed=9)
        m = oracle.StepModel(w.spec(), b, w.in_shape)
        m.params[:] = p0
        loss = m.step(x[rank * b:(rank + 1) * b], y[rank * b:(rank + 1) * b], opt=0, lr=0.0)
        flat = torch.from_numpy(np.concatenate([m.grads, [loss]]).astype(np.float32))
        dist.all_reduce(flat)                                  # the single exchange step
        g = flat[:-1].numpy() / world                          # 1/N scale before the update
        new_p = p0 - w.lr * g                                  # identical SGD on every rank
        uid = [bytes(range(128)) if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        q.put((rank, new_p, float(flat[-1]), uid[0]))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_step_equals_full_batch():
    sys.path[:0] = [os.path.join(ROOT, "oracle")]
    import oracle
    from zillaphp_b200 import configs, synthetic
    if not oracle.available("oracle"):
        oracle.build()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000)
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort(key=lambda t: t[0])
    # reference: one process, whole batch
    w = configs.CNN_SMALL
    x, y = synthetic.batch(w, 16, seed=9)
    p0 = synthetic.init_params(w, seed=9)
    m = oracle.StepModel(w.spec(), 16, w.in_shape)
    m.params[:] = p0
    loss = m.step(x, y, opt=1, lr=w.lr)
    for rank, new_p, loss_sum, uid in res:
        assert uid == bytes(range(128))
        assert abs(loss_sum - loss) / loss < 1e-5
        np.testing.assert_allclose(new_p, m.params, rtol=0, atol=1e-6)
    assert np.array_equal(res[0][1], res[1][1])                # replicas stay identical
