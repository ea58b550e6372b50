"""The allocation-free decode attention entry point.

Some callers cannot allocate device memory while they run: a plugin inside a
host runtime that owns all device memory through its own arena, or a serving
loop that forbids allocation after warm-up (cudaMalloc and cudaFree
synchronize the whole device). accel_b200_attention_decode_noalloc serves
them from a fixed scratch array inside the library. This test calls it
through the C ABI twice in a row and checks each result against the entry
point that takes a caller-owned workspace, within the 1e-4 tolerance of the
other attention tests. It lives in its own file, collected last, and passes
both alone in a fresh process and after the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def test_noalloc_matches_workspace_entry_point(lib, cuda):
    rng = np.random.default_rng(17)
    batch, heads, kvh, hd, max_len, chunk = 6, 9, 3, 64, 700, 64
    lens = torch.tensor([1, 64, 65, 400, 700, 333], dtype=torch.int32, device="cuda")
    kc = torch.from_numpy(rng.standard_normal((batch, kvh, max_len, hd), dtype=np.float32)).cuda()
    vc = torch.from_numpy(rng.standard_normal((batch, kvh, max_len, hd), dtype=np.float32)).cuda()
    q = torch.from_numpy(rng.standard_normal((batch, heads * hd), dtype=np.float32)).cuda()
    row, head, seq = hd, max_len * hd, kvh * max_len * hd
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    need = lib.accel_b200_attention_decode_workspace(batch, heads, kvh, max_len, chunk)
    assert need <= lib.accel_b200_attention_decode_noalloc_limit()
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    want = torch.zeros(batch, heads * hd, device="cuda")
    rc = lib.accel_b200_attention_decode(_p(q), q.stride(0), _p(kc), _p(vc), row, head, seq, _p(lens), batch, heads,
                                         kvh, hd, max_len, chunk, _p(want), want.stride(0), _p(ws), need, None, stream)
    assert rc == 0, lib.accel_b200_last_error()

    outs = []
    for _ in range(2):
        out = torch.full((batch, heads * hd), np.nan, device="cuda")
        rc = lib.accel_b200_attention_decode_noalloc(_p(q), q.stride(0), _p(kc), _p(vc), row, head, seq, _p(lens),
                                                     batch, heads, kvh, hd, max_len, chunk, _p(out), out.stride(0),
                                                     None, stream)
        assert rc == 0, lib.accel_b200_last_error()
        outs.append(out)
    torch.cuda.synchronize()
    ref = want.cpu().numpy()
    for out in outs:
        np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=TOL, atol=TOL)


def test_noalloc_rejects_sizes_beyond_its_scratch(lib, cuda):
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    lens = torch.ones(512, dtype=torch.int32, device="cuda")
    rc = lib.accel_b200_attention_decode_noalloc(_p(out), 0, _p(out), _p(out), 64, 64, 64, _p(lens), 512, 32, 8, 64,
                                                 65536, 64, _p(out), 0, None,
                                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 1
    assert "4 MiB" in lib.accel_b200_last_error().decode()


@pytest.mark.parametrize("batch,heads,kvh,max_len,chunk", [
    (1 << 20, 0, 8, 64, 64),   # no heads: the workspace size reads 0, the call must still be rejected
    (4, 9, 3, 64, 0),          # chunk 0
    (4, 3, 9, 64, 64),         # more kv heads than heads
    (4, 9, -3, 64, 64),        # negative kv heads
    (16385, 1, 1, 1, 64),      # more (sequence, kv head) pairs than arrival counters
    (-1, 9, 3, 64, 64),        # negative batch
])
def test_noalloc_rejects_bad_arguments_before_queueing(lib, cuda, batch, heads, kvh, max_len, chunk):
    """Bad arguments return the error code without touching the scratch: the
    stream stays usable and a correct call afterwards still matches."""
    buf = torch.zeros(64 * 64, dtype=torch.float32, device="cuda")
    lens = torch.ones(8, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.accel_b200_attention_decode_noalloc(_p(buf), 0, _p(buf), _p(buf), 64, 64, 64, _p(lens), batch, heads,
                                                 kvh, 64, max_len, chunk, _p(buf), 0, None, stream)
    assert rc == 1
    torch.cuda.synchronize()
    assert not buf.any()  # nothing was written
