"""The C ABI library loads without a GPU and exports every entry point the
headers in include/ declare; the host-side bindings agree with them. No
device calls."""

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np

from accelep_b200 import synthetic as syn
from accelep_b200._lib import SIGNATURES
from tests.conftest import ROOT

DECL = re.compile(r"ACCEL_B200_API\s+[\w\s\*]+?\b(\w+)\s*\(", re.S)


def declared():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        names.update(DECL.findall(header.read_text()))
    return names


def test_every_declared_symbol_is_exported(lib):
    names = declared()
    assert len(names) > 50
    for name in sorted(names):
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib._name)], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}
    assert names <= exported
    # Nothing but the C ABI and the two C++ entry points of
    # include/accel_b200_device.h leaves the library (hidden visibility
    # elsewhere).
    cxx = {"_ZN10accel_b20016CreateB200DeviceEi", "_ZN10accel_b20014LiveB200AllocsEv"}
    assert cxx <= exported
    assert all(s.startswith(("accel_b200_", "accel_sim_", "accel_llama_")) for s in exported - cxx), sorted(exported)[:20]


def test_bindings_cover_the_headers():
    assert declared() == set(SIGNATURES)


def test_reference_api_names_are_kept():
    """Every accel_sim_* / accel_llama_* entry of the reference header
    (include/accel/sim_api.h:19-116) is declared here under the same name."""
    reference_names = {
        "accel_sim_create", "accel_sim_destroy", "accel_sim_upload", "accel_sim_release", "accel_sim_matmul",
        "accel_sim_reset_stats", "accel_sim_matmuls", "accel_sim_bytes_to_device", "accel_sim_bytes_to_host",
        "accel_sim_last_error", "accel_llama_create", "accel_llama_destroy", "accel_llama_weight",
        "accel_llama_tokenizer", "accel_llama_generate", "accel_llama_encode", "accel_llama_decode",
        "accel_llama_complete", "accel_llama_complete_stream", "accel_llama_forward_ids",
        "accel_llama_logit_max_abs", "accel_llama_reset", "accel_llama_last_error"}
    assert reference_names <= declared()


def test_config_struct_layout():
    from accelep_b200._lib import LlamaConfig

    assert ctypes.sizeof(LlamaConfig) == 36
    assert [f[0] for f in LlamaConfig._fields_] == ["vocab", "hidden", "layers", "heads", "kv_heads", "intermediate",
                                                    "context", "eps", "rope_theta"]


def test_struct_layouts_match_the_header(tmp_path):
    """The ctypes mirrors of the header's structs have the C compiler's size
    and field offsets (a field added to one side and not the other shifts
    what the library reads), and the Python flag constants are the header's."""
    from accelep_b200 import kernels as K
    from accelep_b200._lib import Epilogue, L2Prefetch, Q8Plane

    structs = {"accel_b200_epilogue": Epilogue, "accel_b200_l2_prefetch": L2Prefetch,
               "accel_b200_q8_plane": Q8Plane}
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "accel_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include", str(src), "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        cname, key, value = line.split()
        got[(cname, key)] = int(value)
    for cname, py in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for field, _ in py._fields_:
            assert got[(cname, field)] == getattr(py, field).offset, (cname, field)
    header = (ROOT / "include" / "accel_b200.h").read_text()
    for name, value in (("ACCEL_B200_EP_TRIGGER_AFTER_WAIT", K.EP_TRIGGER_AFTER_WAIT),
                        ("ACCEL_B200_ATTN_CACHE_BEFORE_WAIT", K.ATTN_CACHE_BEFORE_WAIT)):
        assert re.search(rf"#define {name} {value}\b", header), name


def test_library_errors_without_device(lib):
    """On a machine without a GPU the library reports an error instead of
    falling back to a CPU path."""
    import torch

    if torch.cuda.is_available():
        return
    from accelep_b200._lib import LlamaConfig

    cfg = LlamaConfig(64, 16, 1, 2, 1, 32, 8, 1e-5, 1e4)
    assert not lib.accel_llama_create(ctypes.byref(cfg))
    assert b"CUDA" in lib.accel_llama_last_error()
    assert not lib.accel_sim_create()


def test_synthetic_is_deterministic():
    a = syn.llama_weights(syn.TINY_LLAMA, 3)
    b = syn.llama_weights(syn.TINY_LLAMA, 3)
    for key in a:
        assert np.array_equal(a[key], b[key])
    assert a[(syn.W_LM_HEAD, -1)] is a[(syn.W_EMBED, -1)]
    q, s = syn.quantize_rows(a[(syn.W_Q, 0)])
    assert q.dtype == np.int8 and np.abs(q).max() == 127 and s.shape == (a[(syn.W_Q, 0)].shape[0],)
    deq = syn.dequantize_rows(q, s)
    assert np.max(np.abs(deq - a[(syn.W_Q, 0)])) <= np.max(s) / 2 * 1.0001
    x, w, sc = syn.int8_gemm(4, 8, 16, 1)
    assert w.min() >= -127 and w.max() <= 127 and sc.min() >= 1e-3 and sc.max() <= 1e-2
    assert np.array_equal(syn.prompts(syn.SMOLLM2_135M, 2, 5, 1), syn.prompts(syn.SMOLLM2_135M, 2, 5, 1))


def test_dropin_libraries_export_the_reference_entry_points():
    """tests/dropin builds the reference's own runtime, Llama and one-matmul
    API on B200Device (libaccel_dropin.so) and the plugin on it
    (libaccel_ep_b200.so); both load without a GPU and export what their
    callers bind (src/ep.cc:1985-2022 for the plugin)."""
    import pytest

    base = ROOT / "tests" / "_build" / "dropin"
    if not (base / "libaccel_dropin.so").is_file():
        pytest.skip("the drop-in build needs the AccelEP sources (make -C tests/dropin)")
    dropin = ctypes.CDLL(str(base / "libaccel_dropin.so"))
    for name in ("accel_llama_create", "accel_llama_generate", "accel_llama_forward_ids", "accel_sim_matmul",
                 "dropin_execute_matmul_q", "dropin_mlp_block", "dropin_device_name"):
        assert hasattr(dropin, name), name
    if (base / "libaccel_ep_b200.so").is_file():
        ep = ctypes.CDLL(str(base / "libaccel_ep_b200.so"))
        for name in ("CreateEpFactories", "ReleaseEpFactory", "AccelEpKernelMatmuls", "AccelEpBytesToDevice"):
            assert hasattr(ep, name), name
