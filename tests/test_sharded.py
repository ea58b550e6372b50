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
