"""The rest of the decode layer through dianoia's GPU-layer ABI
(lab_gpu_enc_head_norm_rope, _attention, _conv, _copy, _steer), against the
CPU path's arithmetic restated in oracle/lab_oracle.c (shard.dart,
ops.dart, control_vector.dart): bit for bit on seeded inputs (the CPU's
left-to-right double sums are trees here; a double ulp apart, they flip an
f32 output only within that of a rounding boundary, which these inputs do
not meet). Attention is also checked against the reference's own C kernel
(lab_attention, compiled here) within f32 rounding. Shapes: Qwen3-1.7B's
heads (16 query, 8 KV, head_dim 128), decode and prefill chunks, sliding
windows, gated heads, an LFM2-style conv with its history carried across
command buffers, and arguments that do not fit."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


class Bufs:
    """GPU-layer buffers with numpy views of their host mirrors."""

    def __init__(self, L):
        self.L, self.h = L, []

    def make(self, values):
        values = np.ascontiguousarray(values, np.float32)
        h = self.L.lab_gpu_buffer(4 * max(values.size, 1))
        assert h >= 0
        self.h.append(h)
        self.view(h, values.size)[:] = values
        return h

    def view(self, h, count):
        return np.ctypeslib.as_array((ctypes.c_float * count).from_address(self.L.lab_gpu_contents(h)))

    def release(self):
        for h in self.h:
            self.L.lab_gpu_release(h)


@pytest.fixture
def gpu(cuda_lib):
    assert cuda_lib.lab_gpu_init() == 1
    b = Bufs(cuda_lib)
    yield cuda_lib, b
    b.release()


@pytest.mark.parametrize("heads,hd,n,pad", [(16, 128, 1, 0), (8, 128, 5, 1024), (2, 64, 3, 32)])
def test_head_norm_rope(gpu, oracle, heads, hd, n, pad):
    L, B = gpu
    rng = np.random.default_rng(heads + n)
    x_stride = heads * hd + pad         # q of a token, then (say) k and v
    rope_stride = 2 * hd                # full and sliding tables per token
    x = (rng.standard_normal(n * x_stride) * 3).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    rope = rng.uniform(-1, 1, n * rope_stride).astype(np.float32)
    small = np.concatenate([np.zeros(16, np.float32), w])
    hx, hw, hr = B.make(x), B.make(small), B.make(rope)
    L.lab_gpu_begin()
    L.lab_gpu_enc_head_norm_rope(hx, 0, x_stride, hw, 64, hr, 4 * hd, rope_stride, heads, hd, n, 1e-6)
    assert L.lab_gpu_commit(1) == 1
    want = oracle.head_norm_rope(x, x_stride, w, rope[hd:], rope_stride, heads, hd, n, 1e-6)
    assert np.array_equal(bits(B.view(hx, x.size)), bits(want))


@pytest.mark.parametrize("heads,kv,hd,pos,n,window,gated", [
    (16, 8, 128, 0, 1, 0, True),        # the first token
    (16, 8, 128, 777, 1, 0, True),      # decode deep in a sequence
    (16, 8, 128, 40, 6, 0, False),      # a prefill chunk
    (16, 8, 128, 3000, 2, 512, True),   # a sliding layer past its window
    (4, 1, 64, 10, 3, 4, False),
])
def test_attention(gpu, oracle, reference, heads, kv, hd, pos, n, window, gated):
    L, B = gpu
    rng = np.random.default_rng(pos + n + heads)
    q = rng.standard_normal(n * heads * hd).astype(np.float32)
    keys = rng.standard_normal((pos + n) * kv * hd).astype(np.float32)
    values = rng.standard_normal((pos + n) * kv * hd).astype(np.float32)
    gate = rng.standard_normal(n * heads).astype(np.float32) if gated else None
    hq, hk, hv = B.make(q), B.make(keys), B.make(values)
    hg = B.make(gate) if gated else -1
    ho = B.make(np.full(n * heads * hd, np.nan, np.float32))
    L.lab_gpu_begin()
    L.lab_gpu_enc_attention(hq, hk, hv, hg, ho, pos, n, heads, kv, hd, window)
    assert L.lab_gpu_commit(1) == 1
    got = B.view(ho, n * heads * hd).copy()
    want = oracle.attention(q, keys, values, gate, pos, n, heads, kv, hd, window)
    assert np.array_equal(bits(got), bits(want))
    ref = reference.attention(q, keys, values, gate, pos, n, heads, kv, hd, window)
    assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_conv_with_history_across_commits(gpu, oracle):
    L, B = gpu
    rng = np.random.default_rng(8)
    width, k = 1536, 3
    w = rng.standard_normal(width * k).astype(np.float32) * 0.5
    hist0 = np.zeros((k - 1) * width, np.float32)
    hw = B.make(np.concatenate([np.zeros(8, np.float32), w]))
    hh = B.make(hist0)
    hist = hist0
    for n in (5, 1, 1):  # a prefill chunk, then decode steps
        bcx = rng.standard_normal(n * 3 * width).astype(np.float32)
        hb = B.make(bcx)
        hy = B.make(np.full(n * width, np.nan, np.float32))
        L.lab_gpu_begin()
        L.lab_gpu_enc_conv(hb, hw, 32, hh, hy, width, k, n)
        assert L.lab_gpu_commit(1) == 1
        y, hist = oracle.conv(bcx, w, hist, width, k, n)
        assert np.array_equal(bits(B.view(hy, n * width)), bits(y))
        assert np.array_equal(bits(B.view(hh, hist.size)), bits(hist))


@pytest.mark.parametrize("mode,scale", [(0, 1.0), (1, 0.75), (1, 1.0)])
def test_steer_and_copy(gpu, oracle, mode, scale):
    L, B = gpu
    rng = np.random.default_rng(mode + 3)
    rows, cols = 3, 2048
    x = rng.standard_normal(rows * cols).astype(np.float32)
    v = rng.standard_normal(cols).astype(np.float32)
    v /= np.float32(np.linalg.norm(v))
    hx = B.make(x)
    hv = B.make(np.concatenate([np.zeros(4, np.float32), v]))
    hc = B.make(np.zeros(rows * cols + 8, np.float32))
    L.lab_gpu_begin()
    L.lab_gpu_enc_steer(hx, 0, hv, 16, rows, cols, mode, scale)
    L.lab_gpu_enc_copy(hx, 4 * cols, hc, 32, 2 * cols)   # rows 1 and 2, after the steer
    assert L.lab_gpu_commit(1) == 1
    want = oracle.steer(x, v, rows, cols, mode, scale)
    assert np.array_equal(bits(B.view(hx, x.size)), bits(want))
    assert np.array_equal(bits(B.view(hc, rows * cols + 8)[8:8 + 2 * cols]), bits(want[cols:]))


def test_layer_ops_reject_what_does_not_fit(gpu):
    L, B = gpu
    a = B.make(np.zeros(4096, np.float32))
    b = B.make(np.zeros(64, np.float32))
    for record in (
        lambda: L.lab_gpu_enc_head_norm_rope(a, 0, 128, b, 0, a, 0, 128, 1, 130, 1, 1e-6),   # hd odd-sized w
        lambda: L.lab_gpu_enc_head_norm_rope(a, 0, 64, b, 0, a, 0, 128, 1, 128, 1, 1e-6),    # stride < hd
        lambda: L.lab_gpu_enc_head_norm_rope(a, 0, 128, b, 0, a, 0, 128, 1, 257, 1, 1e-6),   # hd > 256
        lambda: L.lab_gpu_enc_attention(a, a, a, -1, a, 0, 1, 3, 2, 64, 0),                   # heads % kv
        lambda: L.lab_gpu_enc_attention(a, b, b, -1, a, 10, 1, 2, 1, 8, 0),                   # keys too short
        lambda: L.lab_gpu_enc_attention(a, a, a, -1, a, 20000, 1, 1, 1, 1, 0),                # too many keys
        lambda: L.lab_gpu_enc_attention(a, a, a, -1, a, 4, 1, 2, 1, 6, 0),                    # hd % 4 != 0
        lambda: L.lab_gpu_enc_conv(a, b, 0, b, a, 64, 17, 1),                                  # k > 16
        lambda: L.lab_gpu_enc_conv(a, b, 0, b, a, 64, 3, 1),                                   # weights short
        lambda: L.lab_gpu_enc_steer(a, 0, b, 0, 1, 128, 1, 1.0),                               # v short
        lambda: L.lab_gpu_enc_steer(a, 0, b, 0, 1, 32, 2, 1.0),                                # no mode 2
        lambda: L.lab_gpu_enc_copy(a, 2, b, 0, 8),                                             # unaligned
        lambda: L.lab_gpu_enc_copy(a, 0, b, 0, 65),                                            # dst short
    ):
        L.lab_gpu_begin()
        record()
        assert L.lab_gpu_commit(1) == 0
    # sliding windows bound the keys a token sees, not the position
    big = B.make(np.zeros(20001 * 8, np.float32))
    L.lab_gpu_begin()
    L.lab_gpu_enc_attention(a, big, big, -1, a, 20000, 1, 1, 1, 8, 512)
    assert L.lab_gpu_commit(1) == 1


def test_attention_over_a_device_only_kv_cache(gpu, oracle):
    """A decode step as GpuForward records it (gpu.dart:1100-1180), less the
    products: q and k normed and rotated in place, the token's k and v copied
    into device-only KV caches (dn_gpu_device_buffer: no host mirror, nothing
    copied per commit), attention over the cached rows. Three tokens in three
    command buffers; every output bit for bit against the CPU path."""
    L, B = gpu
    rng = np.random.default_rng(21)
    heads, kv, hd, max_seq = 4, 2, 64, 8
    q_dim, kv_dim = heads * hd, kv * hd
    keys = L.dn_gpu_device_buffer(4 * max_seq * kv_dim)
    values = L.dn_gpu_device_buffer(4 * max_seq * kv_dim)
    try:
        assert keys >= 0 and values >= 0 and L.lab_gpu_contents(keys) is None
        w = (1 + 0.1 * rng.standard_normal(2 * hd)).astype(np.float32)
        hw = B.make(w)
        qkv = B.make(np.zeros(q_dim + 2 * kv_dim, np.float32))
        rope = B.make(np.zeros(hd, np.float32))
        out = B.make(np.zeros(q_dim, np.float32))
        cache_k = np.zeros(max_seq * kv_dim, np.float32)
        cache_v = np.zeros(max_seq * kv_dim, np.float32)
        for pos in range(3):
            x = rng.standard_normal(q_dim + 2 * kv_dim).astype(np.float32)
            tab = rng.uniform(-1, 1, hd).astype(np.float32)
            B.view(qkv, x.size)[:] = x
            B.view(rope, hd)[:] = tab
            L.lab_gpu_begin()
            L.lab_gpu_enc_head_norm_rope(qkv, 0, q_dim + 2 * kv_dim, hw, 0, rope, 0, hd, heads, hd, 1, 1e-6)
            L.lab_gpu_enc_head_norm_rope(qkv, 4 * q_dim, q_dim + 2 * kv_dim, hw, 4 * hd, rope, 0, hd, kv, hd, 1, 1e-6)
            L.lab_gpu_enc_copy(qkv, 4 * q_dim, keys, 4 * pos * kv_dim, kv_dim)
            L.lab_gpu_enc_copy(qkv, 4 * (q_dim + kv_dim), values, 4 * pos * kv_dim, kv_dim)
            L.lab_gpu_enc_attention(qkv, keys, values, -1, out, pos, 1, heads, kv, hd, 0)
            assert L.lab_gpu_commit(1) == 1
            qn = oracle.head_norm_rope(x[:q_dim], q_dim, w[:hd], tab, hd, heads, hd, 1, 1e-6)
            kn = oracle.head_norm_rope(x[q_dim:q_dim + kv_dim], kv_dim, w[hd:], tab, hd, kv, hd, 1, 1e-6)
            cache_k[pos * kv_dim:(pos + 1) * kv_dim] = kn
            cache_v[pos * kv_dim:(pos + 1) * kv_dim] = x[q_dim + kv_dim:]
            want = oracle.attention(qn, cache_k, cache_v, None, pos, 1, heads, kv, hd, 0)
            assert np.array_equal(bits(B.view(out, q_dim)), bits(want))
            assert np.array_equal(bits(B.view(qkv, q_dim)), bits(qn))
    finally:
        L.lab_gpu_release(keys)
        L.lab_gpu_release(values)


def test_batch_rows_equal_single_calls(gpu):
    """dn_gpu_enc_batch's rows for copy, steer, head norm + RoPE, conv and
    attention (packed small integers) record what the single calls do."""
    L, B = gpu
    rng = np.random.default_rng(5)
    heads, kv, hd, pos = 4, 2, 64, 6
    q_dim, kv_dim = heads * hd, kv * hd
    eps_bits = int(np.array([1e-6], np.float64).view(np.int64)[0])
    scale_bits = int(np.array([0.5], np.float64).view(np.int64)[0])
    x = rng.standard_normal(q_dim + 2 * kv_dim).astype(np.float32)
    cache = rng.standard_normal((pos + 1) * kv_dim).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(2 * hd)).astype(np.float32)
    tab = rng.uniform(-1, 1, hd).astype(np.float32)
    v = rng.standard_normal(q_dim).astype(np.float32)
    width, k = 64, 3
    bcx = rng.standard_normal(2 * 3 * width).astype(np.float32)
    cw = rng.standard_normal(width * k).astype(np.float32)
    results = []
    for batch in (False, True):
        hx, hk, hv, hw, hr = B.make(x), B.make(cache), B.make(cache), B.make(w), B.make(tab)
        ho, hs = B.make(np.zeros(q_dim, np.float32)), B.make(v)
        hb, hcw = B.make(bcx), B.make(cw)
        hh, hy = B.make(np.zeros((k - 1) * width, np.float32)), B.make(np.zeros(2 * width, np.float32))
        L.lab_gpu_begin()
        if batch:
            t = np.array([
                [7, hx, 0, q_dim + 2 * kv_dim, hw, 0, hr, 0, hd, heads | (hd << 16) | (1 << 32), eps_bits],
                [7, hx, 4 * q_dim, q_dim + 2 * kv_dim, hw, 4 * hd, hr, 0, hd, kv | (hd << 16) | (1 << 32), eps_bits],
                [5, hx, 4 * q_dim, hk, 4 * pos * kv_dim, kv_dim, 0, 0, 0, 0, 0],
                [5, hx, 4 * (q_dim + kv_dim), hv, 4 * pos * kv_dim, kv_dim, 0, 0, 0, 0, 0],
                [9, hx, hk, hv, -1, ho, pos, 1, heads, kv, hd | (3 << 32)],
                [6, ho, 0, hs, 0, 1, q_dim, 1, scale_bits, 0, 0],
                [8, hb, hcw, 0, hh, hy, width, k, 2, 0, 0]], np.int64)
            L.dn_gpu_enc_batch(t.ctypes.data, len(t))
        else:
            L.lab_gpu_enc_head_norm_rope(hx, 0, q_dim + 2 * kv_dim, hw, 0, hr, 0, hd, heads, hd, 1, 1e-6)
            L.lab_gpu_enc_head_norm_rope(hx, 4 * q_dim, q_dim + 2 * kv_dim, hw, 4 * hd, hr, 0, hd, kv, hd, 1, 1e-6)
            L.lab_gpu_enc_copy(hx, 4 * q_dim, hk, 4 * pos * kv_dim, kv_dim)
            L.lab_gpu_enc_copy(hx, 4 * (q_dim + kv_dim), hv, 4 * pos * kv_dim, kv_dim)
            L.lab_gpu_enc_attention(hx, hk, hv, -1, ho, pos, 1, heads, kv, hd, 3)
            L.lab_gpu_enc_steer(ho, 0, hs, 0, 1, q_dim, 1, 0.5)
            L.lab_gpu_enc_conv(hb, hcw, 0, hh, hy, width, k, 2)
        assert L.lab_gpu_commit(1) == 1
        results.append([B.view(h, n).copy() for h, n in ((hx, x.size), (hk, cache.size), (ho, q_dim),
                                                          (hy, 2 * width), (hh, (k - 1) * width))])
    for a, b in zip(*results):
        assert np.array_equal(bits(a), bits(b))
    assert np.abs(results[0][2]).max() > 0
