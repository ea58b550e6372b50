"""ctypes binding of the one-matmul C API on the B200 backend.

Same class and methods as the reference binding (serve/sim.py:22-106); the
matrix lives in HBM and the product runs Device::MatMul on a B200Device.
"""

import numpy as np

from ._lib import P_f32, load


class Sim:
    def __init__(self):
        self._lib = load()
        self._sim = self._lib.accel_sim_create()
        if not self._sim:
            raise RuntimeError(self.error() or "create failed")

    def error(self):
        raw = self._lib.accel_sim_last_error()
        return raw.decode() if raw else ""

    def upload(self, values):
        array = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
        buf = self._lib.accel_sim_upload(self._sim, array.ctypes.data_as(P_f32), array.size)
        if not buf:
            raise RuntimeError(self.error() or "upload failed")
        return buf

    def release(self, buf):
        self._lib.accel_sim_release(self._sim, buf)

    def matmul(self, left, weight, n):
        """left is float32 [m, k]; weight an uploaded [k, n] matrix."""
        a = np.ascontiguousarray(left, dtype=np.float32)
        if a.ndim == 1:
            a = a.reshape(1, -1)
        m, k = a.shape
        out = np.empty((m, n), dtype=np.float32)
        status = self._lib.accel_sim_matmul(self._sim, a.ctypes.data_as(P_f32), m, k, weight, n,
                                            out.ctypes.data_as(P_f32))
        if status != 0:
            raise RuntimeError(self.error() or "matmul failed")
        return out

    def reset_stats(self):
        self._lib.accel_sim_reset_stats()

    def matmuls(self):
        return int(self._lib.accel_sim_matmuls())

    def bytes_to_device(self):
        return int(self._lib.accel_sim_bytes_to_device())

    def bytes_to_host(self):
        return int(self._lib.accel_sim_bytes_to_host())

    def close(self):
        if self._sim:
            self._lib.accel_sim_destroy(self._sim)
            self._sim = None

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()
