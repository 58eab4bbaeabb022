"""GPU quantized kernels through the C-ABI against the CPU oracle and the reference's golden vectors.

Mirrors the reference's tests/test_quant.py:119-205 and adds multi-token, row-range, edge and
full-size cases. Bar: dequant bit-exact, activation quantization byte-exact, products bit-exact
to the reference's scalar kernels (K-quants also to its AVX2 kernels).
"""
import ctypes

import numpy as np
import pytest

import oracle
from sardyne_b200 import capi

pytestmark = pytest.mark.gpu
KINDS = oracle.WEIGHT_TYPES
TID = oracle.TYPE_ID


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


def gpu_matmul_q(w, kind, xq, n_tok, n_in, n_out, row0=0, row1=None, out=None):
    row1 = n_out if row1 is None else row1
    if out is None:
        out = np.full((n_tok, n_out), np.nan, np.float32)
    lib().op_matmul_q_rows(ptr(out), ptr(xq), ptr(w), TID[kind], n_tok, n_in, n_out, row0, row1)
    return out


@pytest.mark.parametrize("kind", KINDS)
def test_dequant_bit_exact(golden, kind):
    w, y = golden[f"deq_{kind}_w"], golden[f"deq_{kind}_y"]
    out = np.empty(y.size, np.float32)
    lib().op_row_to_f32(ptr(w), TID[kind], ptr(out), y.size)
    assert np.array_equal(out.view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("vt", ["Q8_0", "Q8_K"])
def test_activation_quantization_byte_exact(golden, vt):
    x = golden["act_x"]
    n_rows, n = x.shape
    out = np.zeros(lib().op_row_size(TID[vt], n) * n_rows, np.uint8)
    lib().op_quantize_rows(TID[vt], ptr(x), ptr(out), n, 0, n_rows)
    assert out.tobytes() == golden[f"act_{vt}"].tobytes()
    # a sub-range of tokens writes only its own rows
    part = np.zeros_like(out)
    lib().op_quantize_rows(TID[vt], ptr(x), ptr(part), n, 2, 5)
    rb = lib().op_row_size(TID[vt], n)
    assert part[2 * rb:5 * rb].tobytes() == out[2 * rb:5 * rb].tobytes() and not part[:2 * rb].any()


@pytest.mark.parametrize("vt", ["Q8_0", "Q8_K"])
@pytest.mark.parametrize("n", [256, 2048, 11008])
def test_activation_quantization_random(vt, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal((7, n)) * rng.uniform(1e-3, 1e3, (7, 1))).astype(np.float32)
    x[3, :] = 0
    x[4, ::7] = 0.5  # exact ties after scaling are likely
    out = np.zeros(lib().op_row_size(TID[vt], n) * 7, np.uint8)
    lib().op_quantize_rows(TID[vt], ptr(x), ptr(out), n, 0, 7)
    assert out.tobytes() == oracle.quantize(x, vt).tobytes()


def same_floats(got, want):
    """Bit-equal, except that NaNs (whose bit patterns differ between the host and the GPU) need
    only sit in the same places."""
    nan = np.isnan(want)
    return np.array_equal(np.isnan(got), nan) and np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


@pytest.mark.parametrize("vt", ["Q8_0", "Q8_K"])
def test_activation_quantization_special_values(vt):
    """Signed zeros, blocks whose inverse scale overflows to infinity (subnormal maxima: the
    reference's conversions then store zeros), values near the float maximum, a negative maximum:
    the bytes of the reference's host (oracle.special_rows, pinned to the reference library)."""
    x = oracle.special_rows(512)
    out = np.zeros(lib().op_row_size(TID[vt], 512) * len(x), np.uint8)
    lib().op_quantize_rows(TID[vt], ptr(x), ptr(out), 512, 0, len(x))
    assert out.tobytes() == oracle.quantize(x, vt).tobytes()


@pytest.mark.parametrize("n_copies", [1, 5])  # 7 tokens: matvec; 35: the tensor-core GEMM
@pytest.mark.parametrize("kind", ["Q4_K", "Q6_K", "Q8_0", "Q4_0"])
def test_products_of_special_rows(kind, n_copies):
    """op_matmul on the special rows (quantized inside the product's kernels) equals the oracle's
    product of the oracle's quantization."""
    x = np.ascontiguousarray(np.tile(oracle.special_rows(512), (n_copies, 1)))
    n_tok, n_in, n_out = x.shape[0], 512, 40
    w = oracle.random_blocks(kind, n_out * n_in // oracle.QK[kind], seed=9)
    got = np.full((n_tok, n_out), np.nan, np.float32)
    lib().op_matmul(ptr(got), ptr(x), ptr(w), TID[kind], n_tok, n_in, n_out)
    want = oracle.matmul_q(w, kind, oracle.quantize(x, oracle.VEC_DOT_TYPE[kind]), n_tok, n_in, n_out)
    assert same_floats(got, want)


@pytest.mark.parametrize("kind", KINDS)
def test_vec_dot_matches_reference(golden, kind):
    w, xq = golden[f"dot_{kind}_w"], golden[f"dot_{kind}_xq"]
    scalar, avx2 = golden[f"dot_{kind}_scalar_avx2"]
    got = np.float32(lib().op_vec_dot_q(TID[kind], ptr(w), ptr(xq), 1024))
    assert got == scalar
    if kind in ("Q4_K", "Q6_K"):
        assert got == avx2


@pytest.mark.parametrize("tag", ["small", "big"])
@pytest.mark.parametrize("kind", KINDS)
def test_matmul_q_rows_golden(golden, tag, kind):
    n_in, n_out, n_tok = golden[f"mm_{tag}_{kind}_shape"].tolist()
    w, xq = golden[f"mm_{tag}_{kind}_w"], golden[f"mm_{tag}_{kind}_xq"]
    out = gpu_matmul_q(w, kind, xq, n_tok, n_in, n_out)
    assert np.array_equal(out, golden[f"mm_{tag}_{kind}_scalar"])
    if kind in ("Q4_K", "Q6_K"):
        assert np.array_equal(out, golden[f"mm_{tag}_{kind}_avx2"])
    parts = np.full_like(out, np.nan)
    for r0, r1 in [(0, 5), (5, 6), (6, n_out)]:
        gpu_matmul_q(w, kind, xq, n_tok, n_in, n_out, r0, r1, out=parts)
    assert np.array_equal(parts, out)


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("n_tok", [1, 2, 3, 4, 5, 7, 8, 9, 13, 33])
def test_matmul_q_rows_tokens(kind, n_tok):
    n_in, n_out = 1024, 37
    w = oracle.random_blocks(kind, n_out * n_in // oracle.QK[kind], seed=n_tok)
    x = np.random.default_rng(n_tok).standard_normal((n_tok, n_in)).astype(np.float32)
    xq = oracle.quantize(x, oracle.VEC_DOT_TYPE[kind])
    assert np.array_equal(gpu_matmul_q(w, kind, xq, n_tok, n_in, n_out),
                          oracle.matmul_q(w, kind, xq, n_tok, n_in, n_out))


@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("n_in,n_out", [(256, 1), (256, 8), (512, 9), (2048, 2048), (576, 24),
                                        (11008, 17), (4096, 300)])
def test_matmul_shapes(kind, n_in, n_out):
    if n_in % oracle.QK[kind]:
        pytest.skip("row not a multiple of the block")
    w = oracle.random_blocks(kind, n_out * n_in // oracle.QK[kind], seed=n_in + n_out)
    x = np.random.default_rng(3).standard_normal((2, n_in)).astype(np.float32)
    xq = oracle.quantize(x, oracle.VEC_DOT_TYPE[kind])
    assert np.array_equal(gpu_matmul_q(w, kind, xq, 2, n_in, n_out), oracle.matmul_q(w, kind, xq, 2, n_in, n_out))


@pytest.mark.parametrize("kind", ["Q8_0", "Q4_0", "Q5_0"])
def test_q0_rows_not_multiple_of_256(kind):
    """SmolLM2's dim 576 = 18 blocks of 32: the 8-block runs end ragged."""
    n_in, n_out = 576, 45
    w = oracle.random_blocks(kind, n_out * n_in // 32, seed=5)
    x = np.random.default_rng(5).standard_normal((3, n_in)).astype(np.float32)
    xq = oracle.quantize(x, "Q8_0")
    assert np.array_equal(gpu_matmul_q(w, kind, xq, 3, n_in, n_out), oracle.matmul_q(w, kind, xq, 3, n_in, n_out))


@pytest.mark.parametrize("kind", ["Q4_0", "Q5_0"])
@pytest.mark.parametrize("n_in,n_tok", [(256, 1), (576, 3)])
def test_q0_tall_matrix(kind, n_in, n_tok):
    """Q4_0 / Q5_0 matrices of LM-head height (80000 rows), a row range that starts inside a row
    group, ragged 8-block runs at 576."""
    n_out = 80000
    w = oracle.random_blocks(kind, n_out * n_in // 32, seed=n_in)
    x = np.random.default_rng(n_in).standard_normal((n_tok, n_in)).astype(np.float32)
    xq = oracle.quantize(x, "Q8_0")
    want = oracle.matmul_q(w, kind, xq, n_tok, n_in, n_out)
    assert np.array_equal(gpu_matmul_q(w, kind, xq, n_tok, n_in, n_out), want)
    got = gpu_matmul_q(w, kind, xq, n_tok, n_in, n_out, row0=3, row1=79000)
    assert np.isnan(got[:, :3]).all() and np.isnan(got[:, 79000:]).all()
    assert np.array_equal(got[:, 3:79000], want[:, 3:79000])


@pytest.mark.parametrize("kind", KINDS)
def test_op_matmul_quantizes_like_the_reference(kind):
    """op_matmul (f32 activations in): quantization + product on the GPU == oracle chain."""
    n_in, n_out, n_tok = 2048, 64, 3
    w = oracle.random_blocks(kind, n_out * n_in // oracle.QK[kind], seed=11)
    x = np.random.default_rng(11).standard_normal((n_tok, n_in)).astype(np.float32)
    out = np.empty((n_tok, n_out), np.float32)
    lib().op_matmul(ptr(out), ptr(x), ptr(w), TID[kind], n_tok, n_in, n_out)
    xq = oracle.quantize(x, oracle.VEC_DOT_TYPE[kind])
    assert np.array_equal(out, oracle.matmul_q(w, kind, xq, n_tok, n_in, n_out))


@pytest.mark.parametrize("kind", ["Q4_K", "Q6_K", "Q5_0"])
def test_op_matmul_into_pinned_output(kind):
    """A page-locked output buffer is written by the kernel itself (no copy after it): same bits,
    and a pageable buffer next to it still gets the copy."""
    import torch
    n_in, n_out, n_tok = 2048, 1000, 2
    w = oracle.random_blocks(kind, n_out * n_in // oracle.QK[kind], seed=13)
    x = np.random.default_rng(13).standard_normal((n_tok, n_in)).astype(np.float32)
    want = oracle.matmul_q(w, kind, oracle.quantize(x, oracle.VEC_DOT_TYPE[kind]), n_tok, n_in, n_out)
    pinned = torch.full((n_tok, n_out), float("nan")).pin_memory()
    for _ in range(2):
        lib().op_matmul(ctypes.c_void_p(pinned.data_ptr()), ptr(x), ptr(w), TID[kind], n_tok, n_in, n_out)
        assert np.array_equal(pinned.numpy(), want)
    plain = np.full((n_tok, n_out), np.nan, np.float32)
    lib().op_matmul(ptr(plain), ptr(x), ptr(w), TID[kind], n_tok, n_in, n_out)
    assert np.array_equal(plain, want)


@pytest.mark.parametrize("kind", KINDS)
def test_registered_weights_read_in_place(kind):
    """Resident weights (sdy_weights_register) give the same bits as staged weights, for any
    row range and for row pointers inside the registered block."""
    n_in, n_out = 2048, 203
    w = oracle.random_blocks(kind, n_out * n_in // oracle.QK[kind], seed=21).reshape(n_out, -1)
    x = np.random.default_rng(21).standard_normal((4, n_in)).astype(np.float32)
    xq = oracle.quantize(x, oracle.VEC_DOT_TYPE[kind])
    want = oracle.matmul_q(w, kind, xq, 4, n_in, n_out)
    assert lib().sdy_weights_register(ptr(w), TID[kind], n_out, n_in) == 0
    try:
        assert np.array_equal(gpu_matmul_q(w, kind, xq, 4, n_in, n_out), want)
        assert np.array_equal(gpu_matmul_q(w, kind, xq, 4, n_in, n_out, 13, 101)[:, 13:101], want[:, 13:101])
        sub = w[50:]  # a pointer into the middle of the registered rows (no copy: same host bytes)
        assert np.array_equal(gpu_matmul_q(sub, kind, xq, 4, n_in, n_out - 50), want[:, 50:])
        row = np.empty(n_in, np.float32)
        lib().op_row_to_f32(ptr(w[77]), TID[kind], ptr(row), n_in)
        assert np.array_equal(row, oracle.dequant(w[77], kind, n_in)[0])
    finally:
        assert lib().sdy_weights_unregister(ptr(w)) == 0


@pytest.mark.parametrize("kind", ["Q4_K", "Q6_K"])
def test_full_size_lm_head(kind):
    """151936 x 2048 (the Qwen LM head, 175-255 MB): resident weights, checked row-exact against
    the oracle on a seeded sample of 3000 rows spread over the whole matrix."""
    n_in, n_out = 2048, 151936
    rng = np.random.default_rng(7)
    w = oracle.random_blocks(kind, n_out * n_in // 256, seed=7).reshape(n_out, -1)
    x = rng.standard_normal((1, n_in)).astype(np.float32)
    xq = oracle.quantize(x, "Q8_K")
    assert lib().sdy_weights_register(ptr(w), TID[kind], n_out, n_in) == 0
    try:
        out = gpu_matmul_q(w, kind, xq, 1, n_in, n_out)
    finally:
        lib().sdy_weights_unregister(ptr(w))
    rows = np.sort(rng.choice(n_out, 3000, replace=False))
    rows[-1] = n_out - 1
    want = np.array([oracle.vec_dot(w[r], kind, xq, n_in) for r in rows], np.float32)
    assert np.array_equal(out[0, rows], want)
    assert np.isfinite(out).all()


def test_f16_conversion_all_values():
    bits = np.arange(1 << 16, dtype=np.uint16)
    out = np.empty(1 << 16, np.float32)
    lib().op_f16_to_f32_n(ptr(bits), ptr(out), bits.size)
    exp = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(exp)
    assert np.array_equal(np.isnan(out), nan)
    assert np.array_equal(out[~nan].view(np.uint32), exp[~nan].view(np.uint32))


def test_f32_to_f16(golden):
    v, ref = golden["f16_in"], golden["f16_out"]
    got = np.array([lib().op_f32_to_f16(float(a)) for a in v], np.uint16)
    assert np.array_equal(got, ref)


def test_errors_are_reported_not_crashing():
    out = np.zeros(4, np.float32)
    w = np.zeros(100, np.uint8)
    lib().op_matmul_q_rows(ptr(out), ptr(w), ptr(w), 3, 1, 32, 1, 0, 1)  # Q4_1: unsupported
    assert b"unsupported" in lib().sdy_last_error()
    lib().sdy_clear_error()


def test_grouped_products_equal_single_launches():
    """sdy_qmatvec_batch_dev: independent products of both K-quant formats, different input widths
    and row counts (ragged groups), in one launch: each equal to its own sdy_qmatvec_dev bit for bit;
    sdy_qmatvec_batch_f32_dev (f32 rows quantized by every CTA) gives the same bits."""
    import torch
    lib_ = lib()
    shapes = [("Q4_K", 300, 2048), ("Q6_K", 1001, 2048), ("Q4_K", 77, 11008), ("Q6_K", 2048, 1024),
              ("Q4_K", 4096, 256), ("Q6_K", 9, 11008)]
    handles, xqs, outs, want, xs = [], [], [], [], []
    try:
        for i, (kind, n_out, n_in) in enumerate(shapes):
            w = oracle.random_blocks(kind, n_out * n_in // 256, seed=50 + i)
            h = lib_.sdy_qmat_upload(ptr(w), TID[kind], n_out, n_in)
            assert h, capi.last_error()
            handles.append(h)
            x = torch.from_numpy(np.random.default_rng(i).standard_normal(n_in).astype(np.float32)).cuda()
            xs.append(x)
            xq = torch.empty(lib_.sdy_xq_bytes(TID["Q8_K"], n_in, 1), dtype=torch.uint8, device="cuda")
            assert lib_.sdy_quantize_rows_dev(TID["Q8_K"], ctypes.c_void_p(x.data_ptr()), 1, n_in,
                                              ctypes.c_void_p(xq.data_ptr()), None) == 0
            xqs.append(xq)
            outs.append(torch.full((n_out,), float("nan"), device="cuda"))
            ref = torch.full((n_out,), float("nan"), device="cuda")
            assert lib_.sdy_qmatvec_dev(h, ctypes.c_void_p(xq.data_ptr()), 1, ctypes.c_void_p(ref.data_ptr()), n_out,
                                        0, n_out, None) == 0
            want.append(ref)
        n = len(shapes)
        arr = lambda vals: (ctypes.c_void_p * len(vals))(*vals)  # noqa: E731
        assert lib_.sdy_qmatvec_batch_dev(n, arr(handles), arr([t.data_ptr() for t in xqs]),
                                          arr([t.data_ptr() for t in outs]), None) == 0, capi.last_error()
        torch.cuda.synchronize()
        for got, ref in zip(outs, want):
            assert torch.equal(got, ref)
        # f32 inputs, every CTA quantizing its row (sdy_qmatvec_batch_f32_dev): the same bits
        outs2 = [torch.full_like(o, float("nan")) for o in outs]
        assert lib_.sdy_qmatvec_batch_f32_dev(n, arr(handles), arr([t.data_ptr() for t in xs]),
                                              arr([t.data_ptr() for t in outs2]), None) == 0, capi.last_error()
        torch.cuda.synchronize()
        for got, ref in zip(outs2, want):
            assert torch.equal(got, ref)
        # more than 8 products are refused
        assert lib_.sdy_qmatvec_batch_dev(9, arr(handles + [handles[0]] * 3), arr([0] * 9), arr([0] * 9), None) == -1
        lib_.sdy_clear_error()
    finally:
        for h in handles:
            lib_.sdy_qmat_free(h)
