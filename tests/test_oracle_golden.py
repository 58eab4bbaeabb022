"""The CPU oracle (oracle/qref.c) against golden vectors produced by the reference itself."""
import numpy as np
import pytest

import oracle

KINDS = oracle.WEIGHT_TYPES


@pytest.mark.parametrize("kind", KINDS)
def test_random_blocks_restatement_matches_reference(golden, kind):
    assert np.array_equal(oracle.random_blocks(kind, 16, seed=0), golden[f"blocks_{kind}_s0"])


@pytest.mark.parametrize("kind", KINDS)
def test_dequant_bit_exact(golden, kind):
    w, y = golden[f"deq_{kind}_w"], golden[f"deq_{kind}_y"]
    got = oracle.dequant(w, kind, y.size)[0]
    assert np.array_equal(got.view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("vt", ["Q8_0", "Q8_K"])
def test_activation_quantization_byte_exact(golden, vt):
    x = golden["act_x"]
    assert oracle.quantize(x, vt).tobytes() == golden[f"act_{vt}"].tobytes()


@pytest.mark.parametrize("kind", KINDS)
def test_vec_dot_equals_reference_scalar(golden, kind):
    w, xq = golden[f"dot_{kind}_w"], golden[f"dot_{kind}_xq"]
    scalar, avx2 = golden[f"dot_{kind}_scalar_avx2"]
    got = np.float32(oracle.vec_dot(w, kind, xq, 1024))
    assert got == scalar  # same integer sums, same fp32 combine order
    if kind in ("Q4_K", "Q6_K"):
        assert got == avx2  # the reference's K-quant scalar and AVX2 paths agree bit for bit
    else:
        assert got == pytest.approx(avx2, rel=1e-5, abs=1e-5)


@pytest.mark.parametrize("tag", ["small", "big"])
@pytest.mark.parametrize("kind", KINDS)
def test_matmul_q_rows(golden, tag, kind):
    n_in, n_out, n_tok = golden[f"mm_{tag}_{kind}_shape"].tolist()
    w, xq = golden[f"mm_{tag}_{kind}_w"], golden[f"mm_{tag}_{kind}_xq"]
    got = oracle.matmul_q(w, kind, xq, n_tok, n_in, n_out)
    assert np.array_equal(got, golden[f"mm_{tag}_{kind}_scalar"])
    parts = np.full_like(got, np.nan)
    for r0, r1 in [(0, 5), (5, 6), (6, n_out)]:
        oracle.matmul_q(w, kind, xq, n_tok, n_in, n_out, r0, r1, out=parts)
    assert np.array_equal(parts, got)


def test_f16_conversions():
    bits = np.arange(1 << 16, dtype=np.uint16)
    exp = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.qref().oq_f16_to_f32(int(b)) for b in bits], np.float32)
    nan = np.isnan(exp)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), exp[~nan].view(np.uint32))


def test_f32_to_f16(golden):
    v, ref = golden["f16_in"], golden["f16_out"]
    got = np.array([oracle.qref().oq_f32_to_f16(float(a)) for a in v], np.uint16)
    assert np.array_equal(got, ref)
    rng = np.random.default_rng(3)
    w = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32)
    got = np.array([oracle.qref().oq_f32_to_f16(float(a)) for a in w], np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(got, w.astype(np.float16).view(np.uint16))


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built here")
@pytest.mark.parametrize("kind", KINDS)
def test_oracle_equals_reference_library_on_fresh_inputs(kind):
    """Beyond the stored vectors: fresh seeds, odd row counts, straight against the reference."""
    ref = oracle.ref()
    ref.op_set_simd(0)
    try:
        for seed in range(3):
            n_in, n_out, n_tok = 1024, 11, 5
            w = oracle.random_blocks(kind, n_out * n_in // oracle.QK[kind], seed=100 + seed)
            x = np.random.default_rng(seed).standard_normal((n_tok, n_in)).astype(np.float32)
            vt = oracle.VEC_DOT_TYPE[kind]
            xq = oracle.quantize(x, vt)
            xq_ref = np.zeros_like(xq)
            ref.op_quantize_rows(oracle.TYPE_ID[vt], x.ctypes.data, xq_ref.ctypes.data, n_in, 0, n_tok)
            assert xq.tobytes() == xq_ref.tobytes()
            want = np.zeros((n_tok, n_out), np.float32)
            ref.op_matmul_q_rows(want.ctypes.data, xq.ctypes.data, w.ctypes.data, oracle.TYPE_ID[kind], n_tok,
                                 n_in, n_out, 0, n_out)
            assert np.array_equal(oracle.matmul_q(w, kind, xq, n_tok, n_in, n_out), want)
    finally:
        ref.op_set_simd(1)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built here")
@pytest.mark.parametrize("vt", ["Q8_0", "Q8_K"])
def test_oracle_quantizers_equal_reference_on_special_values(vt):
    """Signed zeros, blocks whose inverse scale overflows to infinity (subnormal maxima), values near
    the float maximum: the oracle's bytes are the reference library's."""
    x = oracle.special_rows(512)
    want = np.zeros(oracle.row_bytes(vt, 512) * len(x), np.uint8)
    oracle.ref().op_quantize_rows(oracle.TYPE_ID[vt], x.ctypes.data, want.ctypes.data, 512, 0, len(x))
    assert oracle.quantize(x, vt).tobytes() == want.tobytes()
