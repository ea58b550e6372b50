"""Failure detection without a GPU fault: a bounded wait that runs out sets
the timeout bit in its status word and returns, the context stays usable,
and host-side errors map to the reference's error behaviour."""

import numpy as np
import pytest
import torch

from accelep_b200 import kernels as K
from accelep_b200._lib import check

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_context_survives(lib, cuda):
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    check(lib.accel_b200_wait_selftest(K._p(status), K._s()))
    torch.cuda.synchronize()
    assert int(status.item()) & 2  # ACCEL_B200_STATUS_COPY_TIMEOUT
    x = torch.arange(8, dtype=torch.float32, device="cuda")
    y = torch.ones(8, dtype=torch.float32, device="cuda")
    K.residual_add(x, y)
    torch.cuda.synchronize()
    assert x.cpu().tolist() == [float(i + 1) for i in range(8)]


def test_argument_errors_do_not_launch(lib, cuda):
    from accelep_b200._lib import B200Error

    q = torch.zeros(1, 9 * 64, device="cuda")
    with pytest.raises(B200Error, match="bad arguments"):
        K.attention_decode(q, q, q, torch.ones(1, dtype=torch.int32, device="cuda"), 9, 4, 64, 8)
    with pytest.raises(B200Error, match="out of range"):
        check(lib.accel_b200_matmul(None, None, None, -1, 1, 1, None))
    assert "out of range" in lib.accel_b200_last_error().decode()
    np.testing.assert_equal(int(lib.accel_b200_launch_count()) >= 0, True)


def test_peer_barrier_times_out_without_a_peer(lib, cuda):
    """The rank barrier of the fused all-gather waits for a peer that never
    signals (rank 1 of 2 does not exist): the bounded wait runs out (about a
    millisecond here), sets the timeout bit and returns; the context stays
    usable. Rank 1's flag array is a scratch buffer on this GPU."""
    import ctypes

    mine = torch.zeros(2, dtype=torch.int32, device="cuda")
    scratch = torch.zeros(2, dtype=torch.int32, device="cuda")
    flags = (ctypes.c_void_p * 8)(mine.data_ptr(), scratch.data_ptr())
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    check(lib.accel_b200_peer_barrier(flags, K._p(mine), 0, 2, K._p(epoch), 2_000_000, K._p(status), K._s()))
    torch.cuda.synchronize()
    assert int(status.item()) & 2
    assert scratch.cpu().tolist() == [1, 0]  # this rank's signal (epoch 1) landed in the peer's slot 0
    assert int(epoch.item()) == 1
    # Once the peer's signal is there, the next barrier (epoch 2) passes without a timeout.
    mine[1] = 2
    status.zero_()
    check(lib.accel_b200_peer_barrier(flags, K._p(mine), 0, 2, K._p(epoch), 2_000_000, K._p(status), K._s()))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert scratch.cpu().tolist() == [2, 0] and int(epoch.item()) == 2
