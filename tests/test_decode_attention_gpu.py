"""The fused decode step accel_b200_decode_attention (Rope, AppendCache and
attention for one new token per sequence): the cache rows it writes against
accel_b200_rope_append bit for bit, and the attention output against the
CPU checker's Rope + Attention (src/sim_rope.cc, src/sim_attend.cc:9-46)
within 1e-4, over ragged positions (chunk edges, one row, the full context)
and finished rows."""

import numpy as np
import pytest
import torch

from accelep_b200 import kernels as K
from accelep_b200._lib import B200Error

pytestmark = pytest.mark.gpu


def T(a, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a))
    return t.to(dtype).to("cuda") if dtype is not None else t.to("cuda")


def H(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def close(got, want):
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


def tables(ctx, hd, theta=10000.0):
    inv = 1.0 / theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd)
    ang = np.outer(np.arange(ctx, dtype=np.float64), inv)
    ang = np.concatenate([ang, ang], axis=1)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


# C4's decode launch: 32 sequences, 3 kv heads, contexts 512..2048 (the
# kernel splits each (sequence, kv head) over a 4-CTA cluster at this size).
C4_POS = [511, 2047, 1023, 1024, 1279, 1280, 2046, 600, 1900, 767, 1535, 1536, 2000, 513, 1111, 1999,
          640, 704, 1088, 1152, 1408, 1471, 1664, 1727, 1791, 1855, 1920, 1983, 2010, 2040, -1, 1300]


@pytest.mark.parametrize("heads,kvh,ctx,pos", [
    (9, 3, 2048, C4_POS),
    (9, 3, 1300, [0, 63, 64, 700, 1299, -1, 127, 1000]),
    (4, 4, 200, [5, 199, -1, 64]),
    (8, 1, 520, [511, 512, 0]),
])
def test_decode_attention_matches(lib, cuda, orc, heads, kvh, ctx, pos):
    hd = 64
    rng = np.random.default_rng(ctx + heads)
    rows = len(pos)
    pos = np.array(pos, np.int32)
    seq = np.arange(rows, dtype=np.int32)[::-1].copy()  # slots in another order than rows
    qkv = rng.standard_normal((rows, (heads + 2 * kvh) * hd), dtype=np.float32)
    kc = rng.standard_normal((rows, kvh, ctx, hd), dtype=np.float32)
    vc = rng.standard_normal((rows, kvh, ctx, hd), dtype=np.float32)
    cos_t, sin_t = tables(ctx, hd)
    cos_d, sin_d = T(cos_t), T(sin_t)

    # Fused step.
    kc_f, vc_f, qkv_f = T(kc), T(vc), T(qkv)
    out = torch.full((rows, heads * hd), 7.0, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.decode_attention(qkv_f, T(pos), heads, kvh, cos_d, sin_d, kc_f, vc_f, row_seq=T(seq), out=out, status=status)
    got = H(out)
    assert H(status)[0] == 0
    assert np.array_equal(H(qkv_f), qkv)  # the input rows are only read

    # Separate Rope + AppendCache: the same cache bits.
    kc_r, vc_r, qkv_r = T(kc), T(vc), T(qkv)
    K.rope_append(qkv_r, T(seq), T(pos), heads, kvh, hd, cos_d, sin_d, kc_r, vc_r)
    assert np.array_equal(H(kc_f), H(kc_r))
    assert np.array_equal(H(vc_f), H(vc_r))

    kc_after = H(kc_r)
    vc_after = H(vc_r)
    for r in range(rows):
        if pos[r] < 0:
            assert (got[r] == 7.0).all()  # finished: not written
            continue
        p, s = int(pos[r]), int(seq[r])
        q = orc.rope(qkv[r, :heads * hd].copy(), cos_t, sin_t, 1, heads, hd, p)
        k_ref = np.ascontiguousarray(kc_after[s, :, :p + 1].transpose(1, 0, 2))  # [t, kv head, d]
        v_ref = np.ascontiguousarray(vc_after[s, :, :p + 1].transpose(1, 0, 2))
        want = orc.attend(q.reshape(1, heads, hd), k_ref, v_ref, 1, p, heads, kvh, hd)
        close(got[r], want.reshape(-1))


def test_decode_attention_every_split_boundary(lib, cuda, orc):
    """Every length from 1 to 300 in one batch: all chunk and split edges."""
    heads, kvh, hd, ctx = 6, 2, 64, 300
    rng = np.random.default_rng(9)
    pos = np.arange(ctx, dtype=np.int32)
    rows = len(pos)
    qkv = rng.standard_normal((rows, (heads + 2 * kvh) * hd), dtype=np.float32)
    kc = rng.standard_normal((rows, kvh, ctx, hd), dtype=np.float32)
    vc = rng.standard_normal((rows, kvh, ctx, hd), dtype=np.float32)
    cos_t, sin_t = tables(ctx, hd)
    kc_f, vc_f = T(kc), T(vc)
    got = H(K.decode_attention(T(qkv), T(pos), heads, kvh, T(cos_t), T(sin_t), kc_f, vc_f))
    kc_after, vc_after = H(kc_f), H(vc_f)
    for r in range(0, rows, 7):
        p = int(pos[r])
        q = orc.rope(qkv[r, :heads * hd].copy(), cos_t, sin_t, 1, heads, hd, p)
        k_ref = np.ascontiguousarray(kc_after[r, :, :p + 1].transpose(1, 0, 2))
        v_ref = np.ascontiguousarray(vc_after[r, :, :p + 1].transpose(1, 0, 2))
        want = orc.attend(q.reshape(1, heads, hd), k_ref, v_ref, 1, p, heads, kvh, hd)
        close(got[r], want.reshape(-1))


def test_decode_attention_prefetch_same_results(lib, cuda):
    """accel_b200_decode_attention_prefetch (L2 prefetch of other ranges, cache
    rows read evict-first) writes the same outputs and cache bits as
    accel_b200_decode_attention, and leaves the prefetched ranges alone."""
    heads, kvh, hd, ctx = 9, 3, 64, 700
    rng = np.random.default_rng(4)
    pos = np.array([0, 63, 64, 699, -1, 300], np.int32)
    rows = len(pos)
    qkv = rng.standard_normal((rows, (heads + 2 * kvh) * hd), dtype=np.float32)
    kc = rng.standard_normal((rows, kvh, ctx, hd), dtype=np.float32)
    vc = rng.standard_normal((rows, kvh, ctx, hd), dtype=np.float32)
    cos_t, sin_t = tables(ctx, hd)
    weights = [torch.randint(-127, 128, (576, n), dtype=torch.int8, device="cuda") for n in (576, 3072, 100)]
    before = [H(w).copy() for w in weights]
    outs, caches = [], []
    for pf in (None, weights):
        kc_d, vc_d = T(kc), T(vc)
        out = torch.full((rows, heads * hd), 7.0, device="cuda")
        K.decode_attention(T(qkv), T(pos), heads, kvh, T(cos_t), T(sin_t), kc_d, vc_d, out=out, prefetch=pf)
        outs.append(H(out))
        caches.append((H(kc_d), H(vc_d)))
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(caches[0][0], caches[1][0]) and np.array_equal(caches[0][1], caches[1][1])
    for w, b in zip(weights, before):
        assert np.array_equal(H(w), b)
    with pytest.raises(B200Error):  # a range that is not 16-byte aligned
        K.decode_attention(T(qkv), T(pos), heads, kvh, T(cos_t), T(sin_t), T(kc), T(vc), prefetch=[weights[0][0, 1:]])


@pytest.mark.parametrize("n_rows", [8, 32])  # the GEMV and the tensor-core product before the attention
def test_decode_attention_cache_before_wait(lib, cuda, n_rows):
    """The decode step as the engine launches it: a q|k|v product that lets
    the next kernel launch only after its own wait (TRIGGER_AFTER_WAIT), then
    the attention reading the cache before its wait (CACHE_BEFORE_WAIT).
    Outputs and cache bits equal the plain launches'; unknown flag bits are
    rejected."""
    heads, kvh, hd, ctx, hidden = 9, 3, 64, 700, 576
    rng = np.random.default_rng(14)
    pos = np.array([0, 63, 64, 699, -1, 300, 128, 511], np.int32)
    pos = np.concatenate([pos, rng.integers(0, ctx, n_rows - len(pos)).astype(np.int32)])
    rows = len(pos)
    x = rng.standard_normal((rows, hidden), dtype=np.float32)
    w = rng.integers(-127, 128, (hidden, (heads + 2 * kvh) * hd), dtype=np.int8)
    scale = (rng.random((heads + 2 * kvh) * hd, dtype=np.float32) + 0.5) / 256
    kc = rng.standard_normal((rows, kvh, ctx, hd), dtype=np.float32)
    vc = rng.standard_normal((rows, kvh, ctx, hd), dtype=np.float32)
    cos_t, sin_t = tables(ctx, hd)
    x_d, w_d, s_d = T(x), T(w), T(scale)
    outs, caches, qkvs = [], [], []
    for late in (False, True):
        kc_d, vc_d = T(kc), T(vc)
        qkv = torch.zeros(rows, (heads + 2 * kvh) * hd, device="cuda")
        ep = K.make_epilogue(flags=K.EP_TRIGGER_AFTER_WAIT if late else 0)
        K.matmul_q8(x_d, w_d, s_d, epilogue=ep, out=qkv)
        out = torch.full((rows, heads * hd), 7.0, device="cuda")
        K.decode_attention(qkv, T(pos), heads, kvh, T(cos_t), T(sin_t), kc_d, vc_d, out=out,
                           flags=K.ATTN_CACHE_BEFORE_WAIT if late else 0)
        outs.append(H(out))
        qkvs.append(H(qkv))
        caches.append((H(kc_d), H(vc_d)))
    assert np.array_equal(qkvs[0], qkvs[1])
    assert np.array_equal(outs[0], outs[1])
    assert np.array_equal(caches[0][0], caches[1][0]) and np.array_equal(caches[0][1], caches[1][1])
    with pytest.raises(B200Error):
        K.decode_attention(T(qkvs[0]), T(pos), heads, kvh, T(cos_t), T(sin_t), T(kc), T(vc), flags=2)
    with pytest.raises(B200Error):
        K.matmul_q8(x_d, w_d, s_d, epilogue=K.make_epilogue(flags=2))


def test_decode_attention_rejects(lib, cuda):
    q = torch.zeros(2, 9 * 64 + 6 * 64, device="cuda")
    kc = torch.zeros(2, 3, 16, 64, device="cuda")
    pos = torch.zeros(2, dtype=torch.int32, device="cuda")
    cs = torch.zeros(16, 64, device="cuda")
    with pytest.raises(B200Error):
        K.decode_attention(q, pos, 9, 4, cs, cs, kc, kc)  # 9 heads over 4 kv heads
    with pytest.raises(B200Error):
        K.decode_attention(torch.zeros(2, 100, device="cuda"), pos, 9, 3, cs, cs, kc, kc)  # row stride too small


@pytest.mark.parametrize("heads,kvh,counts,pos0", [
    (9, 3, [512, 37, 1, 64, 130], [0, 0, 0, 5, 200]),
    (4, 2, [96, 33], [0, 1000]),
    (4, 4, [65], [3]),
    (8, 2, [40, 7], [0, 60]),
])
def test_prefill_attention_matches(lib, cuda, orc, heads, kvh, counts, pos0):
    """Tiled prefill attention (accel_b200_attention_prefill) against the
    checker's Attention per sequence: ragged prompts, query tiles that end
    mid-tile, continuation at a position offset (ForwardIds after earlier
    rows), and every supported group size."""
    hd = 64
    rng = np.random.default_rng(sum(counts) + heads)
    ctx = max(p + c for p, c in zip(pos0, counts)) + 7
    batch = len(counts)
    first = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int32)
    rows = int(sum(counts))
    q = rng.standard_normal((rows, heads * hd), dtype=np.float32)
    kc = rng.standard_normal((batch, kvh, ctx, hd), dtype=np.float32)
    vc = rng.standard_normal((batch, kvh, ctx, hd), dtype=np.float32)
    got = H(K.attention_prefill(T(q), T(kc), T(vc), T(first), T(np.array(counts, np.int32)),
                                T(np.array(pos0, np.int32)), heads, kvh))
    for b in range(batch):
        n, p = counts[b], pos0[b]
        k_ref = np.ascontiguousarray(kc[b, :, :p + n].transpose(1, 0, 2))
        v_ref = np.ascontiguousarray(vc[b, :, :p + n].transpose(1, 0, 2))
        want = orc.attend(q[first[b]:first[b] + n].reshape(n, heads, hd), k_ref, v_ref, n, p, heads, kvh, hd)
        close(got[first[b]:first[b] + n], want.reshape(n, -1))
