"""Calls into the kernel C ABI with torch CUDA tensors.

torch only provides device memory and the current stream here; every
computation is one of the library's kernels. Used by the parity tests and
the benchmark.
"""

import ctypes

import torch

from ._lib import P_i64, Epilogue, Q8Plane, check, load

ACT = {"none": 0, "relu": 1, "gelu": 2}


def _s(stream=None):
    return ctypes.c_void_p((stream or torch.cuda.current_stream()).cuda_stream)


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def embed(ids, table, seq, id_offset=0, status=None):
    hidden = table.shape[1]
    out = torch.zeros(seq, hidden, dtype=torch.float32, device=table.device)
    check(load().accel_b200_embed(_p(ids), id_offset, _p(table), _p(out), seq, hidden, table.shape[0], _p(status), _s()))
    return out


def rmsnorm(x, w, rows, dim, eps, row_offset=0):
    y = torch.zeros(rows, dim, dtype=torch.float32, device=x.device)
    check(load().accel_b200_rmsnorm(_p(x), _p(w), _p(y), rows, dim, eps, row_offset, _s()))
    return y


def rope(states, cos_t, sin_t, seq, n_heads, head_dim, position):
    check(load().accel_b200_rope(_p(states), _p(cos_t), _p(sin_t), seq, n_heads, head_dim, position, _s()))
    return states


def append_cache(src, cache, seq, position, n_heads, head_dim):
    check(load().accel_b200_append_cache(_p(src), _p(cache), seq, position, n_heads, head_dim, _s()))
    return cache


def attention(q, k, v, seq, position, heads, kv_heads, head_dim):
    out = torch.zeros(seq, heads, head_dim, dtype=torch.float32, device=q.device)
    check(load().accel_b200_attention(_p(q), _p(k), _p(v), _p(out), seq, position, heads, kv_heads, head_dim, _s()))
    return out


def silu_mul(gate, up):
    check(load().accel_b200_silu_mul(_p(gate), _p(up), gate.numel(), _s()))
    return gate


def residual_add(dest, extra):
    check(load().accel_b200_residual_add(_p(dest), _p(extra), dest.numel(), _s()))
    return dest


def sample(logits, vocab, temperature, rng_state, top_k, chosen=None, index=0):
    chosen = chosen if chosen is not None else torch.full((index + 1,), -1, dtype=torch.int32, device=logits.device)
    check(load().accel_b200_sample(_p(logits), _p(chosen), index, vocab, temperature, _p(rng_state), top_k, _s()))
    return chosen


def argmax_rows(logits):
    rows, vocab = logits.shape
    chosen = torch.full((rows,), -1, dtype=torch.int32, device=logits.device)
    check(load().accel_b200_argmax_rows(_p(logits), rows, vocab, logits.stride(0), _p(chosen), 1, 0, _s()))
    return chosen


def sample_rows(logits, temperature, rng_states, top_k):
    rows, vocab = logits.shape
    chosen = torch.full((rows,), -1, dtype=torch.int32, device=logits.device)
    check(load().accel_b200_sample_rows(_p(logits), rows, vocab, logits.stride(0), _p(chosen), 1, 0, temperature,
                                        _p(rng_states), top_k, _s()))
    return chosen


def matmul_exact(a, b):
    m, k = a.shape
    n = b.shape[1]
    c = torch.full((m, n), 7.0, dtype=torch.float32, device=a.device)
    check(load().accel_b200_matmul(_p(a), _p(b), _p(c), m, k, n, _s()))
    return c


def transpose(src):
    rows, cols = src.shape
    dst = torch.zeros(cols, rows, dtype=torch.float32, device=src.device)
    check(load().accel_b200_transpose(_p(src), _p(dst), rows, cols, _s()))
    return dst


def gemm_epilogue(c, alpha, bias, bias_shape, beta, act):
    m, n = c.shape
    shape = (ctypes.c_int64 * max(1, len(bias_shape)))(*bias_shape)
    check(load().accel_b200_gemm_epilogue(_p(c), m, n, alpha, _p(bias), ctypes.cast(shape, P_i64),
                                          len(bias_shape) if bias is not None else 0, beta, ACT[act], _s()))
    return c


EP_TRIGGER_AFTER_WAIT = 1  # ACCEL_B200_EP_TRIGGER_AFTER_WAIT
ATTN_CACHE_BEFORE_WAIT = 1  # ACCEL_B200_ATTN_CACHE_BEFORE_WAIT


def make_epilogue(alpha=1.0, beta=0.0, bias=None, bias_strides=(0, 0), act="none", residual=None, row_sq=None,
                  flags=0):
    """row_sq: a float64 [m, ceil(n / 128)] tensor that receives each row's
    sums of squares of the outputs per 128-column block. flags: launch
    options (EP_TRIGGER_AFTER_WAIT)."""
    ep = Epilogue()
    ep.alpha, ep.beta = alpha, beta
    ep.bias = 0 if bias is None else bias.data_ptr()
    ep.bias_row_stride, ep.bias_col_stride = bias_strides
    ep.act = ACT[act]
    ep.residual = 0 if residual is None else residual.data_ptr()
    ep.residual_ld = 0 if residual is None else residual.stride(0)
    ep.row_sq = 0 if row_sq is None else row_sq.data_ptr()
    ep.row_sq_ld = 0 if row_sq is None else row_sq.stride(0)
    ep.flags = flags
    # The struct holds raw addresses: keep the tensors alive with it.
    ep._keep = (bias, residual, row_sq)
    return ep


class Workspace:
    """Grows a zero-filled device byte buffer on demand (the kernels keep
    arrival counters in it and leave them zero)."""

    def __init__(self, device="cuda"):
        self.device = device
        self.buf = None

    def get(self, nbytes):
        if nbytes == 0:
            return None
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        return self.buf


def set_q8_path(path):
    """0: by shape (tensor cores where eligible), 1: CUDA cores only."""
    check(load().accel_b200_set_q8_path(path))


_WS = {}


def _workspace(device, nbytes):
    ws = _WS.setdefault(str(device), Workspace(device))
    return ws.get(nbytes)


def matmul_q8(a, q, scale, zero=None, axis=1, epilogue=None, out=None, offset=0, workspace=None):
    """a [m, k] fp32, q int8 holding a [k, n] plane (at `offset`)."""
    lib = load()
    m, k = a.shape
    n = q.shape[-1]
    c = out if out is not None else torch.zeros(m, n, dtype=torch.float32, device=a.device)
    plane = Q8Plane(q.data_ptr(), scale.data_ptr(), 0 if zero is None else zero.data_ptr(), offset, axis)
    need = lib.accel_b200_matmul_q8_workspace(m, k, n)
    ws = workspace if workspace is not None else _workspace(a.device, need)
    check(lib.accel_b200_matmul_q8(_p(a), a.stride(0), ctypes.byref(plane), _p(c), c.stride(0), m, k, n,
                                   None if epilogue is None else ctypes.byref(epilogue), _p(ws),
                                   0 if ws is None else ws.numel(), _s()))
    return c


def matmul_q8_silu(gate_up, q, scale, axis=1, epilogue=None, out=None, workspace=None):
    """SiluMul(gate_up[:, :inter], gate_up[:, inter:]) @ dequant(q); q holds a
    [inter, n] plane."""
    lib = load()
    m, two_inter = gate_up.shape
    inter = two_inter // 2
    n = q.shape[-1]
    c = out if out is not None else torch.zeros(m, n, dtype=torch.float32, device=gate_up.device)
    plane = Q8Plane(q.data_ptr(), scale.data_ptr(), 0, 0, axis)
    need = lib.accel_b200_matmul_q8_silu_workspace(m, inter, n)
    ws = workspace if workspace is not None else _workspace(gate_up.device, need)
    check(lib.accel_b200_matmul_q8_silu(_p(gate_up), gate_up.stride(0), inter, ctypes.byref(plane), _p(c), c.stride(0),
                                        m, n, None if epilogue is None else ctypes.byref(epilogue), _p(ws),
                                        0 if ws is None else ws.numel(), _s()))
    return c


def matmul_q8_rmsnorm(x, gamma, eps, q, scale, axis=1, epilogue=None, out=None, workspace=None):
    """RmsNorm(x[:, :k]) @ dequant(q); q holds a [k, n] plane (x's row stride
    may be wider than k)."""
    lib = load()
    m = x.shape[0]
    k, n = q.shape
    c = out if out is not None else torch.zeros(m, n, dtype=torch.float32, device=x.device)
    plane = Q8Plane(q.data_ptr(), scale.data_ptr(), 0, 0, axis)
    need = lib.accel_b200_matmul_q8_rmsnorm_workspace(m, k, n)
    ws = workspace if workspace is not None else _workspace(x.device, need)
    check(lib.accel_b200_matmul_q8_rmsnorm(_p(x), x.stride(0), _p(gamma), eps, ctypes.byref(plane), _p(c), c.stride(0),
                                           m, k, n, None if epilogue is None else ctypes.byref(epilogue), _p(ws),
                                           0 if ws is None else ws.numel(), _s()))
    return c


def matmul_q8_rmsnorm_stats(x, row_sq, gamma, eps, q, scale, axis=1, epilogue=None, out=None, workspace=None):
    """RmsNorm(x[:, :k]) @ dequant(q) with each row's sum of squares given as
    row_sq [m, blocks] (float64 partial sums, added in order)."""
    lib = load()
    m = x.shape[0]
    k, n = q.shape
    c = out if out is not None else torch.zeros(m, n, dtype=torch.float32, device=x.device)
    plane = Q8Plane(q.data_ptr(), scale.data_ptr(), 0, 0, axis)
    need = lib.accel_b200_matmul_q8_rmsnorm_workspace(m, k, n)
    ws = workspace if workspace is not None else _workspace(x.device, need)
    check(lib.accel_b200_matmul_q8_rmsnorm_stats(_p(x), x.stride(0), _p(row_sq), row_sq.stride(0), row_sq.shape[1],
                                                 _p(gamma), eps, ctypes.byref(plane), _p(c), c.stride(0), m, k, n,
                                                 None if epilogue is None else ctypes.byref(epilogue), _p(ws),
                                                 0 if ws is None else ws.numel(), _s()))
    return c


def pair_gate_up(gate_up, inter):
    """Columns [gate (inter) | up (inter)] of a weight (or a scale vector) in
    the 64-column pairs accel_b200_matmul_q8_rmsnorm_silu_pairs reads: block
    t holds gate columns 64t .. 64t + 63, then the same up columns."""
    lead = gate_up.shape[:-1]
    g = gate_up[..., :inter].reshape(*lead, inter // 64, 64)
    u = gate_up[..., inter:].reshape(*lead, inter // 64, 64)
    return torch.stack([g, u], dim=-2).reshape(*lead, 2 * inter).contiguous()


def matmul_q8_rmsnorm_silu_pairs(x, gamma, eps, q, scale, row_sq=None, axis=1, out=None, workspace=None):
    """SiluMul(gate, up) of RmsNorm(x[:, :k]) @ dequant(q), q's columns in
    64-column gate|up pairs (pair_gate_up); the result has n / 2 columns.
    row_sq: optional [m, blocks] float64 sums of squares of x's rows."""
    lib = load()
    m = x.shape[0]
    k, n = q.shape
    c = out if out is not None else torch.zeros(m, n // 2, dtype=torch.float32, device=x.device)
    plane = Q8Plane(q.data_ptr(), scale.data_ptr(), 0, 0, axis)
    need = lib.accel_b200_matmul_q8_rmsnorm_workspace(m, k, n)
    ws = workspace if workspace is not None else _workspace(x.device, need)
    sq_ld, sq_n = (row_sq.stride(0), row_sq.shape[1]) if row_sq is not None else (0, 0)
    check(lib.accel_b200_matmul_q8_rmsnorm_silu_pairs(_p(x), x.stride(0), _p(row_sq), sq_ld, sq_n, _p(gamma), eps,
                                                      ctypes.byref(plane), _p(c), c.stride(0), m, k, n, _p(ws),
                                                      0 if ws is None else ws.numel(), _s()))
    return c


def matmul_f32(a, b, epilogue=None, out=None):
    lib = load()
    m, k = a.shape
    n = b.shape[1]
    c = out if out is not None else torch.zeros(m, n, dtype=torch.float32, device=a.device)
    need = lib.accel_b200_matmul_f32_workspace(m, k, n)
    ws = _workspace(a.device, need)
    check(lib.accel_b200_matmul_f32(_p(a), a.stride(0), _p(b), _p(c), c.stride(0), m, k, n,
                                    None if epilogue is None else ctypes.byref(epilogue), _p(ws),
                                    0 if ws is None else ws.numel(), _s()))
    return c


def attention_decode(q, k_cache, v_cache, lens, heads, kv_heads, head_dim, max_len, chunk=64, head_major=False,
                     workspace=None, status=None):
    """q [B, heads * head_dim]. Caches [B, max_len, kv_heads, head_dim] (the
    reference layout) or, with head_major, [B, kv_heads, max_len, head_dim]."""
    lib = load()
    batch = q.shape[0]
    out = torch.zeros(batch, heads * head_dim, dtype=torch.float32, device=q.device)
    need = lib.accel_b200_attention_decode_workspace(batch, heads, kv_heads, max_len, chunk)
    ws = workspace if workspace is not None else torch.zeros(need, dtype=torch.uint8, device=q.device)
    if head_major:
        row, head, seq = head_dim, max_len * head_dim, kv_heads * max_len * head_dim
    else:
        row, head, seq = kv_heads * head_dim, head_dim, max_len * kv_heads * head_dim
    check(lib.accel_b200_attention_decode(_p(q), q.stride(0), _p(k_cache), _p(v_cache), row, head, seq, _p(lens), batch,
                                          heads, kv_heads, head_dim, max_len, chunk, _p(out), out.stride(0), _p(ws),
                                          ws.numel(), _p(status), _s()))
    return out


def rope_append(qkv, row_seq, row_pos, heads, kv_heads, head_dim, cos_t, sin_t, k_cache, v_cache):
    """Rope + AppendCache over fused q|k|v rows (queries rotated in place).
    Caches head-major [slots, kv_heads, context, head_dim]."""
    ctx = k_cache.shape[2]
    check(load().accel_b200_rope_append(_p(qkv), qkv.stride(0), _p(row_seq), _p(row_pos), qkv.shape[0], heads,
                                        kv_heads, head_dim, _p(cos_t), _p(sin_t), _p(k_cache), _p(v_cache),
                                        kv_heads * ctx * head_dim, ctx * head_dim, head_dim, _s()))


def decode_attention(qkv, row_pos, heads, kv_heads, cos_t, sin_t, k_cache, v_cache, row_seq=None, out=None,
                     status=None, prefetch=None, flags=0):
    """Fused decode step (Rope, AppendCache, attention) over un-rotated q|k|v
    rows; caches head-major [slots, kv_heads, context, 64]. prefetch: up to
    four contiguous device tensors to bring into L2 meanwhile (a hint).
    flags: launch options (ATTN_CACHE_BEFORE_WAIT)."""
    rows, ctx = qkv.shape[0], k_cache.shape[2]
    if out is None:
        out = torch.zeros(rows, heads * 64, dtype=torch.float32, device=qkv.device)
    args = (_p(qkv), qkv.stride(0), _p(row_seq), _p(row_pos), rows, heads, kv_heads, 64, _p(cos_t), _p(sin_t), ctx,
            _p(k_cache), _p(v_cache), kv_heads * ctx * 64, ctx * 64, _p(out), out.stride(0), _p(status))
    if prefetch is None and flags == 0:
        check(load().accel_b200_decode_attention(*args, _s()))
    else:
        from ._lib import L2Prefetch
        pf = L2Prefetch()
        for i, t in enumerate(prefetch or []):
            pf.ptr[i] = t.data_ptr()
            pf.bytes[i] = t.numel() * t.element_size()
        pf.count = len(prefetch or [])
        pf.flags = flags
        check(load().accel_b200_decode_attention_prefetch(*args, ctypes.byref(pf), _s()))
    return out


def attention_prefill(q, k_cache, v_cache, first, count, pos0, heads, kv_heads, out=None, max_rows=None):
    """Tiled causal prefill attention. q [rows, heads * 64] (roped); caches
    head-major [slots, kv_heads, context, 64]; first/count/pos0 int32 [batch]
    device tensors."""
    rows = q.shape[0]
    ctx = k_cache.shape[2]
    if out is None:
        out = torch.zeros(rows, heads * 64, dtype=torch.float32, device=q.device)
    batch = first.shape[0]
    if max_rows is None:
        max_rows = int(count.max().item()) if batch else 0
    check(load().accel_b200_attention_prefill(_p(q), q.stride(0), _p(k_cache), _p(v_cache), kv_heads * ctx * 64,
                                              ctx * 64, _p(out), out.stride(0), _p(first), _p(count), _p(pos0), batch,
                                              max_rows, heads, kv_heads, 64, _s()))
    return out


def attention_decode_workspace(batch, heads, kv_heads, max_len, chunk=64, device="cuda"):
    """A zeroed workspace for attention_decode (its counters start at zero)."""
    need = load().accel_b200_attention_decode_workspace(batch, heads, kv_heads, max_len, chunk)
    return torch.zeros(need, dtype=torch.uint8, device=device)
