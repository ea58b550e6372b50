"""B200 backend for AccelEP's device calls.

The product is the C ABI library libaccelep_b200.so (headers in include/):
hand-written sm_100a kernels behind AccelEP's named device calls, the
accel::Device implementation B200Device, and the reference's
accel_sim_* / accel_llama_* C API. This package loads it and mirrors the
reference's Python bindings (serve/sim.py, serve/llama.py).
"""

from ._lib import LIB_PATH, B200Error, load  # noqa: F401

__all__ = ["LIB_PATH", "B200Error", "load"]
