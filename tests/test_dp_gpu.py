"""The data-parallel runner on two GPUs (NCCL): zilla_dp_unique_id /
zilla_dp_attach, one process per GPU, each rank training its half of the
global batch (GPU; skipped with fewer than two GPUs).

* fp32 engine: after two steps, every rank's weights equal the oracle's
  full-batch steps within 1e-4 normwise (only the order of the cross-rank
  gradient sum differs), and the loss slot carries the global loss sum.
* bf16 engine: the ranks end bit-identical to each other, and within the
  engine's stated tolerance (2e-2 normwise) of one GPU training the whole
  batch.
"""
import os
import sys

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


def _rank(rank, world, name, batch, precision, steps, uid_q, out_q, graph=False):
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
    import torch
    torch.cuda.set_device(rank)
    from zillaphp_b200 import configs, synthetic
    from zillaphp_b200.net import Net, dp_unique_id
    try:
        w = configs.WORKLOADS[name]
        b = batch // world
        net = Net(w, batch=b, precision=precision)
        net.set_params(synthetic.init_params(w, seed=21))
        if world > 1:
            if rank == 0:
                uid = dp_unique_id()
                for _ in range(world - 1):
                    uid_q.put(uid)
            else:
                uid = uid_q.get(timeout=60)
            net.dp_attach(rank, world, uid)
        if graph:
            net.set_graph(True)
        losses = []
        for s in range(steps):
            x, y = synthetic.batch(w, batch, seed=21, step=s)
            losses.append(net.step_host(x[rank * b:(rank + 1) * b], y[rank * b:(rank + 1) * b]))
        net.device_status()
        out_q.put((rank, net.params(), losses, None))
        net.close()
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, None, None, repr(e)))


def _run(world, name, batch, precision, steps, graph=False):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, name, batch, precision, steps, uid_q, out_q, graph))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            rank, params, losses, err = out_q.get(timeout=240)
            assert err is None, f"rank {rank}: {err}"
            res[rank] = (params, losses)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.timeout(600)
def test_two_gpu_fp32_step_matches_full_batch_oracle():
    sys.path[:0] = [os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]
    import npref
    import oracle
    from zillaphp_b200 import configs, synthetic
    name, batch, steps = "cnn_1x8_pool_fc", 64, 2
    res = _run(2, name, batch, 0, steps)
    w = configs.WORKLOADS[name]
    ref = oracle.StepModel(w.spec(), batch, w.in_shape, kind="oracle")
    ref.params[:] = synthetic.init_params(w, seed=21)
    ref_losses = []
    for s in range(steps):
        x, y = synthetic.batch(w, batch, seed=21, step=s)
        ref_losses.append(ref.step(x, y, opt=w.optimizer, lr=w.lr))
    assert np.array_equal(res[0][0], res[1][0]), "ranks diverged"
    assert npref.normwise(res[0][0], ref.params) < 1e-4
    for got, want in zip(res[0][1], ref_losses):
        assert abs(got - want) / abs(want) < 1e-5, (got, want)


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.timeout(600)
def test_two_gpu_bf16_step_matches_one_gpu():
    sys.path[:0] = [os.path.join(ROOT, "tests")]
    import npref
    name, batch, steps = "large_cnn", 256, 2
    two = _run(2, name, batch, 1, steps)
    one = _run(1, name, batch, 1, steps)
    assert np.array_equal(two[0][0], two[1][0]), "ranks diverged"
    assert npref.normwise(two[0][0], one[0][0]) < 2e-2
    for got, want in zip(two[0][1], one[0][1]):
        assert abs(got - want) / abs(want) < 2e-2, (got, want)


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.timeout(600)
def test_two_phase_exchange_equals_one_phase():
    """ZB_PEER_TWO_PHASE=1 (the late layers' exchange and update on a side stream beside the
    fused conv backward) does the same per-element arithmetic as the one-phase update: the
    ranks' parameters and losses are bit-identical to the default step's."""
    name, batch, steps = "large_cnn", 256, 3
    one = _run(2, name, batch, 1, steps)
    os.environ["ZB_PEER_TWO_PHASE"] = "1"
    try:
        two = _run(2, name, batch, 1, steps)
    finally:
        del os.environ["ZB_PEER_TWO_PHASE"]
    assert np.array_equal(two[0][0], two[1][0]), "ranks diverged"
    assert np.array_equal(two[0][0], one[0][0]), "two-phase update differs from one-phase"
    assert two[0][1] == one[0][1], (two[0][1], one[0][1])


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.timeout(600)
def test_peer_step_graphs_equal_plain_steps():
    """zilla_net_set_graph under data parallelism: each step's kernels, the peer-memory exchange
    and update among them, are captured per exchange buffer (step parity) and replayed with the
    step's number and Adam arguments.  Six steps (two plain, two captured, two replayed per
    parity) leave both ranks bit-identical to the plain run's parameters and losses."""
    name, batch, steps = "large_cnn", 256, 6
    plain = _run(2, name, batch, 1, steps)
    graph = _run(2, name, batch, 1, steps, graph=True)
    assert np.array_equal(graph[0][0], graph[1][0]), "ranks diverged"
    assert np.array_equal(graph[0][0], plain[0][0]), "graph replay differs from the plain steps"
    assert graph[0][1] == plain[0][1], (graph[0][1], plain[0][1])
