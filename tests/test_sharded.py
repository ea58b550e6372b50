"""The N-sharded C5 product (accelep_b200/sharded.py) on two CPU ranks over
gloo: the gathered Y equals the unsharded product column for column, with
the CPU checker as each rank's local product. The GPU form of the same code
(NCCL, CUDA kernels) runs in bench.py at N > 1."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, m, k, n, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from oracle.oracle import Restated

        from accelep_b200 import sharded
        from accelep_b200 import synthetic as syn

        orc = Restated()
        x, w, s = syn.int8_gemm(m, k, n, 7)

        def cpu_product(xt, wt, st, out):
            out.copy_(torch.from_numpy(orc.execute_matmul_q(xt.numpy(), wt.numpy(), st.numpy())))
            return out

        ws, ss = sharded.shard_columns(torch.from_numpy(w), torch.from_numpy(s), rank, world)
        layer = sharded.ShardedQ8Linear(ws, ss, product=cpu_product)
        y = layer(torch.from_numpy(x))
        if rank == 0:
            np.save(out_path, y.numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m,k,n", [(1, 256, 64), (5, 96, 128)])
def test_sharded_gather_equals_unsharded(tmp_path, m, k, n):
    from oracle.oracle import Restated

    from accelep_b200 import synthetic as syn

    out = str(tmp_path / "y.npy")
    mp.start_processes(_worker, args=(2, _free_port(), m, k, n, out), nprocs=2, join=True, start_method="spawn")
    got = np.load(out)
    x, w, s = syn.int8_gemm(m, k, n, 7)
    want = Restated().execute_matmul_q(x, w, s)
    assert np.array_equal(got, want)


def test_shard_columns_rejects_ragged():
    from accelep_b200 import sharded

    with pytest.raises(ValueError):
        sharded.shard_columns(torch.zeros(4, 6, dtype=torch.int8), torch.zeros(6), 0, 4)


def _failure_worker(rank, world, port, how, deadline, out_dir):
    """Rank 1 fails before the all-gather (`how`: "exit" leaves the process,
    "stall" sleeps past the deadline); rank 0 must end its call with
    CollectiveFailed within the deadline and abort the communicator."""
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from accelep_b200 import sharded

    def cpu_product(xt, wt, st, out):
        out.copy_((xt.double() @ (wt.double() * st.double())).float())
        return out

    w = torch.randint(-127, 128, (16, 8), dtype=torch.int8)
    s = torch.rand(8) * 1e-2
    ws, ss = sharded.shard_columns(w, s, rank, world)
    layer = sharded.ShardedQ8Linear(ws, ss, product=cpu_product, deadline=deadline)
    x = torch.randn(2, 16)
    # One healthy call first: the deadline path gathers like the plain path.
    y = layer(x)
    np.save(os.path.join(out_dir, f"healthy_{rank}.npy"), y.numpy())
    if rank == 1:
        if how == "exit":
            os._exit(0)  # the host process of rank 1 is gone
        time.sleep(deadline + 6)  # alive but stalled past the deadline
        os._exit(0)
    t0 = time.monotonic()
    try:
        layer(x)
        outcome = "completed"
    except sharded.CollectiveFailed:
        outcome = "failed"
    elapsed = time.monotonic() - t0
    try:
        layer(x)
        again = "completed"
    except sharded.CollectiveFailed:
        again = "failed"
    np.save(os.path.join(out_dir, "rank0.npy"), np.array([outcome == "failed", elapsed, again == "failed", layer.aborted]))
    os._exit(0)


@pytest.mark.parametrize("how", ["exit", "stall"])
def test_gather_deadline_aborts_on_a_lost_rank(tmp_path, how):
    """SURVEY's host-side failure case for the N-sharded all-gather: a rank
    that dies (or stalls) before the collective; the survivor's call fails
    with CollectiveFailed within the deadline and the communicator is
    aborted, so the next call fails at once instead of hanging."""
    deadline = 2.0
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failure_worker, args=(r, 2, port, how, deadline, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join()
    y0, y1 = np.load(tmp_path / "healthy_0.npy"), np.load(tmp_path / "healthy_1.npy")
    assert np.array_equal(y0, y1)
    failed, elapsed, again, aborted = np.load(tmp_path / "rank0.npy")
    assert failed and again and aborted
    assert elapsed < deadline + 3.0, elapsed


def test_deadline_needs_the_nccl_mode():
    from accelep_b200 import sharded

    with pytest.raises(ValueError):
        sharded.ShardedQ8Linear(torch.zeros(4, 2, dtype=torch.int8), torch.zeros(2), mode="fused", deadline=1.0)
