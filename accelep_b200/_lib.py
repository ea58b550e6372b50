"""Loads libaccelep_b200.so and declares its C signatures.

The library is built in-tree (python -m accelep_b200.build, or
__graft_entry__.build()). There is no fallback: if the library is missing or
cannot load, every entry point raises.
"""

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libaccelep_b200.so"

c_i32, c_i64, c_u32, c_f32, c_int, c_sz, c_vp = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_float,
                                                 ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p)
P_f32 = ctypes.POINTER(ctypes.c_float)
P_i32 = ctypes.POINTER(ctypes.c_int32)
P_i64 = ctypes.POINTER(ctypes.c_int64)
P_i8 = ctypes.POINTER(ctypes.c_int8)
P_u32 = ctypes.POINTER(ctypes.c_uint32)


class Q8Plane(ctypes.Structure):
    """accel_b200_q8_plane (include/accel_b200.h)."""

    _fields_ = [("q", c_vp), ("scale", c_vp), ("zero", c_vp), ("offset", c_i64), ("axis", c_i32)]


class Epilogue(ctypes.Structure):
    """accel_b200_epilogue (include/accel_b200.h)."""

    _fields_ = [("alpha", c_f32), ("beta", c_f32), ("bias", c_vp), ("bias_row_stride", c_i64),
                ("bias_col_stride", c_i64), ("act", c_i32), ("residual", c_vp), ("residual_ld", c_i64),
                ("row_sq", c_vp), ("row_sq_ld", c_i64), ("flags", c_i32)]


class L2Prefetch(ctypes.Structure):
    """accel_b200_l2_prefetch (include/accel_b200.h)."""

    _fields_ = [("ptr", c_vp * 4), ("bytes", c_i64 * 4), ("count", c_i32), ("flags", c_i32)]


class LlamaConfig(ctypes.Structure):
    """AccelLlamaConfig (include/accel_b200_llama.h)."""

    _fields_ = [("vocab", c_i32), ("hidden", c_i32), ("layers", c_i32), ("heads", c_i32), ("kv_heads", c_i32),
                ("intermediate", c_i32), ("context", c_i32), ("eps", c_f32), ("rope_theta", c_f32)]


P_plane = ctypes.POINTER(Q8Plane)
P_ep = ctypes.POINTER(Epilogue)

# name -> (restype, argtypes). Device pointers and streams travel as c_void_p.
SIGNATURES = {
    "accel_b200_last_error": (ctypes.c_char_p, []),
    "accel_b200_launch_count": (c_i64, []),
    "accel_b200_embed": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "accel_b200_rmsnorm": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_f32, c_i64, c_vp]),
    "accel_b200_rope": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "accel_b200_append_cache": (c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "accel_b200_attention": (c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp]),
    "accel_b200_silu_mul": (c_int, [c_vp, c_vp, c_i64, c_vp]),
    "accel_b200_residual_add": (c_int, [c_vp, c_vp, c_i64, c_vp]),
    "accel_b200_sample": (c_int, [c_vp, c_vp, c_i64, c_i64, c_f32, c_vp, c_i32, c_vp]),
    "accel_b200_argmax_rows": (c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp]),
    "accel_b200_matmul": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "accel_b200_transpose": (c_int, [c_vp, c_vp, c_i64, c_i64, c_vp]),
    "accel_b200_gemm_epilogue": (c_int, [c_vp, c_i64, c_i64, c_f32, c_vp, P_i64, c_i32, c_f32, c_i32, c_vp]),
    "accel_b200_matmul_q8_workspace": (c_sz, [c_i64, c_i64, c_i64]),
    "accel_b200_set_q8_path": (c_int, [c_i32]),
    "accel_b200_matmul_q8": (c_int, [c_vp, c_i64, P_plane, c_vp, c_i64, c_i64, c_i64, c_i64, P_ep, c_vp, c_sz, c_vp]),
    "accel_b200_matmul_q8_peers": (c_int, [c_vp, c_i64, P_plane, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_i32, P_ep,
                                           c_vp, c_sz, c_vp]),
    "accel_b200_peer_barrier": (c_int, [c_vp, c_vp, c_i32, c_i32, c_vp, c_i64, c_vp, c_vp]),
    "accel_b200_matmul_q8_silu_workspace": (c_sz, [c_i64, c_i64, c_i64]),
    "accel_b200_matmul_q8_silu": (c_int, [c_vp, c_i64, c_i64, P_plane, c_vp, c_i64, c_i64, c_i64, P_ep, c_vp, c_sz,
                                          c_vp]),
    "accel_b200_matmul_q8_rmsnorm_workspace": (c_sz, [c_i64, c_i64, c_i64]),
    "accel_b200_matmul_q8_rmsnorm": (c_int, [c_vp, c_i64, c_vp, c_f32, P_plane, c_vp, c_i64, c_i64, c_i64, c_i64,
                                             P_ep, c_vp, c_sz, c_vp]),
    "accel_b200_matmul_q8_rmsnorm_stats": (c_int, [c_vp, c_i64, c_vp, c_i64, c_i32, c_vp, c_f32, P_plane, c_vp,
                                                   c_i64, c_i64, c_i64, c_i64, P_ep, c_vp, c_sz, c_vp]),
    "accel_b200_matmul_q8_rmsnorm_silu_pairs": (c_int, [c_vp, c_i64, c_vp, c_i64, c_i32, c_vp, c_f32, P_plane, c_vp,
                                                        c_i64, c_i64, c_i64, c_i64, c_vp, c_sz, c_vp]),
    "accel_b200_matmul_f32_workspace": (c_sz, [c_i64, c_i64, c_i64]),
    "accel_b200_matmul_f32": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, P_ep, c_vp, c_sz, c_vp]),
    "accel_b200_rope_append": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp,
                                       c_i64, c_i64, c_i64, c_vp]),
    "accel_b200_attention_rows": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp,
                                          c_i64, c_i32, c_i32, c_i32, c_vp]),
    "accel_b200_attention_prefill": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp,
                                             c_i32, c_i32, c_i32, c_i32, c_i32, c_vp]),
    "accel_b200_attention_decode_workspace": (c_sz, [c_i32, c_i32, c_i32, c_i32, c_i32]),
    "accel_b200_attention_decode": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i32, c_i32, c_i32,
                                            c_i32, c_i32, c_i32, c_vp, c_i64, c_vp, c_sz, c_vp, c_vp]),
    "accel_b200_attention_decode_noalloc_limit": (c_sz, []),
    "accel_b200_attention_decode_noalloc": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i32, c_i32,
                                                    c_i32, c_i32, c_i32, c_i32, c_vp, c_i64, c_vp, c_vp]),
    "accel_b200_decode_attention": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp, c_i32,
                                            c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp]),
    "accel_b200_decode_attention_prefetch": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i32, c_i32, c_i32, c_vp, c_vp,
                                                     c_i32, c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp,
                                                     ctypes.POINTER(L2Prefetch), c_vp]),
    "accel_b200_silu_mul_rows": (c_int, [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "accel_b200_sample_rows": (c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_f32, c_vp, c_i32, c_vp]),
    "accel_b200_greedy_step": (c_int, [c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp, c_i32,
                                       c_i32, c_vp, c_vp, c_i32, c_vp]),
    "accel_b200_gather_rows": (c_int, [c_vp, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp]),
    "accel_b200_max_abs_diff": (c_int, [c_vp, c_vp, c_i64, c_vp, c_vp]),
    "accel_b200_wait_selftest": (c_int, [c_vp, c_vp]),
    # The reference's one-matmul API.
    "accel_sim_create": (c_vp, []),
    "accel_sim_destroy": (None, [c_vp]),
    "accel_sim_upload": (c_vp, [c_vp, P_f32, c_i64]),
    "accel_sim_release": (None, [c_vp, c_vp]),
    "accel_sim_matmul": (c_int, [c_vp, P_f32, c_i64, c_i64, c_vp, c_i64, P_f32]),
    "accel_sim_reset_stats": (None, []),
    "accel_sim_matmuls": (c_i64, []),
    "accel_sim_bytes_to_device": (c_i64, []),
    "accel_sim_bytes_to_host": (c_i64, []),
    "accel_sim_last_error": (ctypes.c_char_p, []),
    # The reference's Llama API and its additions.
    "accel_llama_create": (c_vp, [ctypes.POINTER(LlamaConfig)]),
    "accel_llama_destroy": (None, [c_vp]),
    "accel_llama_weight": (c_int, [c_vp, c_i32, c_i32, P_f32, c_i64, c_i64]),
    "accel_llama_weight_q8": (c_int, [c_vp, c_i32, c_i32, P_i8, P_f32, c_i64, c_i64]),
    "accel_llama_tokenizer": (c_int, [c_vp, ctypes.c_char_p]),
    "accel_llama_generate": (c_int, [c_vp, P_i32, c_i32, c_i32, c_i32, c_f32, c_u32, c_i32, P_i32, P_i32]),
    "accel_llama_generate_batch": (c_int, [c_vp, P_i32, P_i32, c_i32, c_i32, c_i32, c_f32, c_u32, P_u32, c_i32,
                                           P_i32, P_i32]),
    "accel_llama_forward_ids": (c_int, [c_vp, P_i32, c_i32, c_i32]),
    "accel_llama_logit_max_abs": (c_int, [c_vp, P_f32, c_i32, P_f32]),
    "accel_llama_logits": (c_int, [c_vp, P_f32, c_i32]),
    "accel_llama_cache_rows": (c_int, [c_vp, c_i32, c_i32, c_i32, c_i32, P_f32]),
    "accel_llama_reset": (None, [c_vp]),
    "accel_llama_last_error": (ctypes.c_char_p, []),
    "accel_llama_stream": (c_vp, [c_vp]),
    "accel_llama_encode": (c_int, [c_vp, ctypes.c_char_p, c_i32, P_i32, c_i32, P_i32]),
    "accel_llama_decode": (c_int, [c_vp, P_i32, c_i32, c_i32, ctypes.c_char_p, c_i32, P_i32]),
    "accel_llama_complete": (c_int, [c_vp, ctypes.c_char_p, c_i32, c_i32, c_i32, c_f32, c_u32, c_i32,
                                     ctypes.c_char_p, c_i32, P_i32, P_i32, c_i32, P_i32, P_i32]),
    "accel_llama_complete_stream": (c_int, [c_vp, ctypes.c_char_p, c_i32, c_i32, c_i32, c_f32, c_u32, c_i32,
                                            ctypes.c_char_p, c_i32, P_i32, P_i32, c_i32, P_i32, P_i32, c_vp, c_vp]),
}

_LIB = None


def load():
    """Returns the loaded library; raises if it has not been built."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.is_file():
            raise FileNotFoundError(f"{LIB_PATH} is missing: build it with `python -m accelep_b200.build`")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _LIB = lib
    return _LIB


class B200Error(RuntimeError):
    """A nonzero status from the kernel ABI."""


def check(rc, lib=None):
    if rc != 0:
        lib = lib or load()
        raise B200Error(f"status {rc}: {lib.accel_b200_last_error().decode()}")
