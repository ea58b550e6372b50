"""The one-matmul C API (accel_sim_*, the reference's serve/sim.py binding)
on the B200 device: the reference's own check (tests/test_serve.py:239-251:
a 2x3 @ 3x4 product with the matmul counter at 1 and bytes moved to the
device), bit-exact products on larger shapes, and its error reporting."""

import numpy as np
import pytest

from accelep_b200.sim import Sim

pytestmark = pytest.mark.gpu


def test_matmul_matches_numpy(lib, cuda):
    left = np.arange(6, dtype=np.float32).reshape(2, 3)
    weight = np.arange(12, dtype=np.float32).reshape(3, 4)
    with Sim() as sim:
        sim.reset_stats()
        uploaded = sim.upload(weight)
        got = sim.matmul(left, uploaded, 4)
        sim.release(uploaded)
        assert sim.matmuls() == 1
        assert sim.bytes_to_device() > 0
        assert sim.bytes_to_host() == got.nbytes
    assert np.array_equal(got, left @ weight)


def test_matmul_bits_and_errors(lib, cuda, orc):
    rng = np.random.default_rng(2)
    a = rng.standard_normal((5, 700), dtype=np.float32)
    b = rng.standard_normal((700, 33), dtype=np.float32)
    with Sim() as sim:
        w = sim.upload(b)
        assert np.array_equal(sim.matmul(a, w, 33), orc.matmul(a, b))  # PackedMatMul's rounding
        assert np.array_equal(sim.matmul(a[0], w, 33)[0], orc.matmul(a[:1], b)[0])
        with pytest.raises(RuntimeError):
            sim.matmul(a, w, 34)  # the uploaded matrix is smaller than k * n
        assert sim.error()
        sim.release(w)
