"""The fp32 kernels behind the op_* hooks (reference tests/test_runtime.py:47-155), on the GPU.

Besides the reference's tolerances against NumPy, the row-split and scalar-order checks pin the
reference's operation order: dot products with four accumulators and separately rounded steps.
"""
import numpy as np
import pytest

import oracle
from sardyne_b200 import capi
from sardyne_b200.gguf_writer import f32_to_bf16

pytestmark = pytest.mark.gpu
F32, F16, BF16 = 0, 1, 30


def lib():
    return capi.lib()


def ptr(a):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


@pytest.fixture(autouse=True)
def no_errors():
    capi.lib().sdy_clear_error()
    yield
    capi.check()


def scalar_dot(x, w):
    """The reference's scalar dot (csrc/ops.c:155-167) in float32 arithmetic."""
    x, w = x.astype(np.float32), w.astype(np.float32)
    s = [np.float32(0)] * 4
    n = len(x)
    i = 0
    while i + 4 <= n:
        for k in range(4):
            s[k] = np.float32(s[k] + np.float32(x[i + k] * w[i + k]))
        i += 4
    while i < n:
        s[0] = np.float32(s[0] + np.float32(x[i] * w[i]))
        i += 1
    return np.float32(np.float32(s[0] + s[1]) + np.float32(s[2] + s[3]))


@pytest.mark.parametrize("wtype", [F32, F16, BF16], ids=["f32", "f16", "bf16"])
@pytest.mark.parametrize("n_tok", [1, 2, 3, 5, 9])
@pytest.mark.parametrize("n_in", [67, 96])
def test_matmul(wtype, n_tok, n_in):
    rng = np.random.default_rng(0)
    n_out = 45
    x = rng.standard_normal((n_tok, n_in)).astype(np.float32)
    w32 = rng.standard_normal((n_out, n_in)).astype(np.float32)
    if wtype == F16:
        w = w32.astype(np.float16)
        w_ref = w.astype(np.float32)
    elif wtype == BF16:
        w = f32_to_bf16(w32)
        w_ref = (w.astype(np.uint32) << 16).view(np.float32)
    else:
        w, w_ref = w32, w32
    out = np.empty((n_tok, n_out), np.float32)
    lib().op_matmul(ptr(out), ptr(x), ptr(w), wtype, n_tok, n_in, n_out)
    np.testing.assert_allclose(out, x @ w_ref.T, rtol=1e-5, atol=1e-5)
    assert out[n_tok - 1, 7] == scalar_dot(x[n_tok - 1], w_ref[7])
    parts = np.full_like(out, np.nan)
    for r0, r1 in [(0, 10), (10, 30), (30, n_out)]:
        lib().op_matmul_rows(ptr(parts), ptr(x), ptr(w), wtype, n_tok, n_in, n_out, r0, r1)
    assert np.array_equal(parts, out)


@pytest.mark.parametrize("n", [1, 7, 8, 64, 100])
def test_dot_and_axpy(n):
    rng = np.random.default_rng(4)
    a, b = rng.standard_normal((2, n)).astype(np.float32)
    got = lib().op_dot_f32(ptr(a), ptr(b), n)
    assert np.float32(got) == scalar_dot(a, b)
    y = rng.standard_normal(n).astype(np.float32)
    expected = (y + (np.float32(0.5) * a).astype(np.float32)).astype(np.float32)
    lib().op_axpy(ptr(y), 0.5, ptr(a), n)
    assert np.array_equal(y, expected)


def test_rmsnorm_softmax_silu():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(300) * 5).astype(np.float32)
    w = rng.standard_normal(300).astype(np.float32)
    out = np.empty_like(x)
    lib().op_rmsnorm(ptr(out), ptr(x), ptr(w), x.size, 1e-5)
    scale = np.float32(1.0 / np.sqrt(np.sum(x.astype(np.float64) ** 2) / x.size + np.float64(np.float32(1e-5))))
    assert np.array_equal(out, (x * scale).astype(np.float32) * w)

    s = np.array([1000.0, 1001.0, -50.0, 3.0], np.float32)
    e = oracle.expf(s - s.max())
    expected = e * np.float32(1.0 / e.astype(np.float64).sum())
    lib().op_softmax(ptr(s), s.size)
    assert np.array_equal(s, expected)

    g = np.array([-100.0, -1.0, 0.0, 2.0, 50.0], np.float32)
    up = np.array([3.0, 2.0, 1.0, -1.0, 0.5], np.float32)
    ex = oracle.expf(-g)
    expected = (g / (np.float32(1) + ex)).astype(np.float32) * up
    lib().op_silu_mul(ptr(g), ptr(up), g.size)
    np.testing.assert_array_equal(g, expected)


@pytest.mark.parametrize("interleaved", [False, True], ids=["neox", "interleaved"])
def test_rope(interleaved):
    n_pos, hd, n_heads, theta = 40, 16, 3, 10000.0
    cos = np.empty((n_pos, hd // 2), np.float32)
    sin = np.empty_like(cos)
    lib().op_rope_table(ptr(cos), ptr(sin), n_pos, hd, theta)
    inv = 1.0 / theta ** (np.arange(0, hd, 2, dtype=np.float64) / hd)
    ang = np.arange(n_pos, dtype=np.float64)[:, None] * inv[None, :]
    np.testing.assert_array_equal(cos, np.cos(ang).astype(np.float32))
    np.testing.assert_array_equal(sin, np.sin(ang).astype(np.float32))
    x = np.random.default_rng(2).standard_normal((n_heads, hd)).astype(np.float32)
    pos = 33
    c, s = cos[pos], sin[pos]
    ia = np.arange(0, hd, 2) if interleaved else np.arange(hd // 2)
    ib = ia + 1 if interleaved else ia + hd // 2
    want = x.copy()
    want[:, ia] = x[:, ia] * c - x[:, ib] * s
    want[:, ib] = x[:, ia] * s + x[:, ib] * c
    row_c, row_s = np.ascontiguousarray(c), np.ascontiguousarray(s)
    lib().op_rope(ptr(x), n_heads, hd, ptr(row_c), ptr(row_s), int(interleaved))
    assert np.array_equal(x, want)


def test_attention_gqa():
    rng = np.random.default_rng(3)
    n_head, n_kv_head, hd, stride, n_kv = 6, 2, 8, 20, 13
    q = rng.standard_normal((n_head, hd)).astype(np.float32)
    kc = rng.standard_normal((n_kv_head, stride, hd)).astype(np.float32)
    vc = rng.standard_normal((n_kv_head, stride, hd)).astype(np.float32)
    out = np.empty_like(q)
    scores = np.empty(stride, np.float32)
    lib().op_attention(ptr(out), ptr(q), ptr(kc), ptr(vc), n_head, n_kv_head, hd, n_kv, stride, ptr(scores))
    n_rep = n_head // n_kv_head
    want = np.empty_like(q)
    scale = np.float32(1) / np.sqrt(np.float32(hd))
    for h in range(n_head):
        k, v = kc[h // n_rep, :n_kv], vc[h // n_rep, :n_kv]
        sc = np.array([scalar_dot(q[h], k[j]) * scale for j in range(n_kv)], np.float32)
        e = oracle.expf(sc - sc.max())
        p = e * np.float32(1.0 / e.astype(np.float64).sum())
        acc = np.zeros(hd, np.float32)
        for j in range(n_kv):
            acc = (acc + (p[j] * v[j]).astype(np.float32)).astype(np.float32)
        want[h] = acc
    assert np.array_equal(out, want)


def attention_model(q, kc, vc, n_kv_head, n_kv):
    """The reference's op_attention (csrc/ops.c:405-423, scalar kernels) in float32 NumPy steps:
    four-accumulator dots, libm's expf, sequential double sum, and the weighted V sum one key at a
    time."""
    n_head, hd = q.shape
    n_rep = n_head // n_kv_head
    scale = np.float32(1) / np.sqrt(np.float32(hd))
    out = np.empty_like(q)
    for h in range(n_head):
        k, v = kc[h // n_rep, :n_kv], vc[h // n_rep, :n_kv]
        s = np.zeros((4, n_kv), np.float32)
        for i in range(0, hd, 4):
            for a in range(4):
                s[a] = s[a] + q[h, i + a] * k[:, i + a]
        sc = ((s[0] + s[1]) + (s[2] + s[3])) * scale
        e = oracle.expf(sc - sc.max())
        p = e * np.float32(1.0 / sum(e.astype(np.float64).tolist()))
        acc = np.zeros(hd, np.float32)
        for j in range(n_kv):
            acc = acc + p[j] * v[j]
        out[h] = acc
    return out


@pytest.mark.parametrize("n_head,n_kv_head,hd,stride,n_kv", [
    (16, 2, 128, 1024, 1), (16, 2, 128, 1024, 7), (16, 2, 128, 1024, 777), (32, 4, 128, 4096, 4096),
    (9, 3, 64, 2048, 300), (8, 8, 128, 516, 515), (32, 1, 64, 256, 200), (16, 2, 256, 600, 599),
    (16, 2, 128, 1023, 500), (4, 4, 80, 64, 50), (16, 2, 128, 8192, 3000)])
def test_attention_vs_reference(n_head, n_kv_head, hd, stride, n_kv):
    """The cluster kernel's shapes (head_dim a multiple of 32, stride a multiple of 4; probabilities
    pushed to every CTA, or pulled in chunks when a long stride does not fit) and the per-head
    fallback's: bit-exact against the operation-order model and against the reference's own
    op_attention (both sides take glibc's expf: the GPU restates its method, expf_ref.h)."""
    if not oracle.ref_available():
        pytest.skip("reference library not built")
    rng = np.random.default_rng(n_kv)
    q = (rng.standard_normal((n_head, hd)) * 0.5).astype(np.float32)
    kc = rng.standard_normal((n_kv_head, stride, hd)).astype(np.float32)
    vc = rng.standard_normal((n_kv_head, stride, hd)).astype(np.float32)
    out, want = np.empty_like(q), np.empty_like(q)
    scores = np.empty(stride, np.float32)  # the reference's work buffer: kept alive across the calls
    lib().op_attention(ptr(out), ptr(q), ptr(kc), ptr(vc), n_head, n_kv_head, hd, n_kv, stride, ptr(scores))
    assert np.array_equal(out, attention_model(q, kc, vc, n_kv_head, n_kv))
    ref = oracle.ref()
    ref.op_set_simd(0)
    ref.op_attention(ptr(want), ptr(q), ptr(kc), ptr(vc), n_head, n_kv_head, hd, n_kv, stride, ptr(scores))
    assert np.array_equal(out, want)


def test_add():
    rng = np.random.default_rng(0)
    a = rng.standard_normal(1023).astype(np.float32)
    b = rng.standard_normal(1023).astype(np.float32)
    out = np.empty_like(a)
    lib().engine_add_f32(a, b, out, a.size)
    np.testing.assert_array_equal(out, a + b)


def test_simd_selection():
    assert lib().op_set_simd(0) == 0 and lib().op_simd() == 0
    assert lib().op_set_simd(1) == 1 and lib().op_simd() == 1
