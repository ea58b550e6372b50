"""The N-sharded C5 product on two GPUs (one rank each, NCCL): the NCCL
all-gather and the fused product + all-gather over peer memory give the same
Y bit for bit on every rank (the same local kernel computes each column
block), within tolerance of the unsharded product (a narrower N changes the
split-K plan, so the summation order differs), over repeated calls (the
fused mode alternates two Y buffers and advances the barrier epoch). Needs
two GPUs; skipped otherwise."""

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, m, k, n, out_dir):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))
    try:
        from accelep_b200 import kernels as K
        from accelep_b200 import sharded
        from accelep_b200 import synthetic as syn

        x, w, s = syn.int8_gemm(m, k, n, 31)
        xt = torch.from_numpy(x).cuda()
        ws, ss = sharded.shard_columns(torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda(), rank, world)
        full = K.matmul_q8(xt, torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda())
        for mode in ("nccl", "fused"):
            layer = sharded.ShardedQ8Linear(ws, ss, mode=mode)
            for it in range(3):
                y = layer(xt * (it + 1))
                torch.cuda.synchronize()
                np.save(os.path.join(out_dir, f"{mode}_{rank}_{it}.npy"), y.cpu().numpy())
            if layer.status is not None:
                np.save(os.path.join(out_dir, f"status_{rank}.npy"), layer.status.cpu().numpy())
        if rank == 0:
            for it in range(3):
                np.save(os.path.join(out_dir, f"full_{it}.npy"), K.matmul_q8(xt * (it + 1), torch.from_numpy(w).cuda(),
                                                                          torch.from_numpy(s).cuda()).cpu().numpy())
        del full
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m,k,n", [(1, 4096, 4096), (300, 1024, 2048)])
def test_sharded_two_gpus(tmp_path, m, k, n):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _free_port(), m, k, n, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for it in range(3):
        full = np.load(tmp_path / f"full_{it}.npy")
        ref = np.load(tmp_path / f"nccl_0_{it}.npy")
        for mode in ("nccl", "fused"):
            for rank in range(2):
                assert np.array_equal(np.load(tmp_path / f"{mode}_{rank}_{it}.npy"), ref), (mode, rank, it)
        np.testing.assert_allclose(ref, full, rtol=1e-4, atol=1e-3 * (it + 1))
    for rank in range(2):
        assert int(np.load(tmp_path / f"status_{rank}.npy")[0]) == 0


def _lost_rank_worker(rank, world, port, deadline, out_dir):
    """NCCL form of the host-side failure case: rank 1 leaves between calls
    (its stream drained, nothing in flight); rank 0's next gather, waited for
    with a deadline, ends with CollectiveFailed and ncclCommAbort."""
    import datetime
    import time

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=30))
    from accelep_b200 import sharded
    from accelep_b200 import synthetic as syn

    x, w, s = syn.int8_gemm(4, 512, 256, 3)
    ws, ss = sharded.shard_columns(torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda(), rank, world)
    layer = sharded.ShardedQ8Linear(ws, ss, mode="nccl", deadline=deadline)
    y = layer(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"healthy_{rank}.npy"), y.cpu().numpy())
    if rank == 1:
        torch.cuda.synchronize()
        os._exit(0)
    time.sleep(1.0)  # rank 1 is gone before this rank's next launch
    t0 = time.monotonic()
    try:
        layer(torch.from_numpy(x).cuda())
        failed = False
    except sharded.CollectiveFailed:
        failed = True
    np.save(os.path.join(out_dir, "rank0.npy"), np.array([failed, time.monotonic() - t0, layer.aborted]))
    os._exit(0)


def test_nccl_gather_deadline_on_a_lost_rank(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    deadline = 3.0
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_lost_rank_worker, args=(r, 2, port, deadline, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            p.join()
    assert np.array_equal(np.load(tmp_path / "healthy_0.npy"), np.load(tmp_path / "healthy_1.npy"))
    failed, elapsed, aborted = np.load(tmp_path / "rank0.npy")
    assert failed and aborted
    assert elapsed < deadline + 3.0, elapsed
