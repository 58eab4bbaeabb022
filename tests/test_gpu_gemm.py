"""The tensor-core prefill GEMM (qgemm.cu) through the C-ABI: op_matmul_q_rows with 32 or more
tokens of Q4_K/Q6_K weights (Q8_K activations) and of Q8_0/Q4_0/Q5_0 weights (Q8_0 activations;
rows whose block count is not a multiple of the kernel's 4-block step, as SmolLM2's 576). Bar:
bit-exact to the reference's scalar kernels (the CPU oracle), like the matvec, over ragged row and
token tiles and row sub-ranges."""
import numpy as np
import pytest

import oracle
from sardyne_b200 import capi

pytestmark = pytest.mark.gpu
TID = oracle.TYPE_ID


def ptr(a):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


@pytest.fixture(autouse=True)
def no_errors():
    capi.lib().sdy_clear_error()
    yield
    capi.check()
    assert capi.lib().sdy_kernel_status() == 0


BLOCK32 = ("Q8_0", "Q4_0", "Q5_0")


def run(kind, n_tok, n_in, n_out, row0=0, row1=None, seed=0):
    row1 = n_out if row1 is None else row1
    be = 32 if kind in BLOCK32 else 256
    w = oracle.random_blocks(kind, n_out * n_in // be, seed=seed)
    x = np.random.default_rng(seed).standard_normal((n_tok, n_in)).astype(np.float32)
    xq = oracle.quantize(x, "Q8_0" if kind in BLOCK32 else "Q8_K")
    out = np.full((n_tok, n_out), np.nan, np.float32)
    capi.lib().op_matmul_q_rows(ptr(out), ptr(xq), ptr(w), TID[kind], n_tok, n_in, n_out, row0, row1)
    want = np.full((n_tok, n_out), np.nan, np.float32)
    oracle.matmul_q(w, kind, xq, n_tok, n_in, n_out, row0, row1, out=want)
    return out, want


@pytest.mark.parametrize("kind", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("n_tok,n_in,n_out", [(32, 256, 8), (40, 512, 200), (128, 2048, 128), (129, 1024, 300),
                                              (300, 2048, 257), (64, 11008, 136)])
def test_gemm_bit_exact(kind, n_tok, n_in, n_out):
    out, want = run(kind, n_tok, n_in, n_out, seed=n_tok + n_out)
    assert np.array_equal(out, want, equal_nan=True)


@pytest.mark.parametrize("kind", ["Q4_K", "Q6_K"])
def test_gemm_row_range(kind):
    """Rows outside [row0, row1) stay untouched; a range starting inside a row group."""
    out, want = run(kind, 150, 1024, 400, row0=13, row1=333, seed=7)
    assert np.isnan(out[:, :13]).all() and np.isnan(out[:, 333:]).all()
    assert np.array_equal(out, want, equal_nan=True)


@pytest.mark.parametrize("kind", BLOCK32)
@pytest.mark.parametrize("n_tok,n_in,n_out", [(32, 32, 8), (40, 96, 200), (128, 576, 128), (129, 576, 1536),
                                              (300, 1536, 257), (64, 11008, 136)])
def test_gemm32_bit_exact(kind, n_tok, n_in, n_out):
    out, want = run(kind, n_tok, n_in, n_out, seed=n_tok + n_out)
    assert np.array_equal(out, want, equal_nan=True)


@pytest.mark.parametrize("kind", BLOCK32)
def test_gemm32_row_range(kind):
    out, want = run(kind, 150, 576, 400, row0=13, row1=333, seed=7)
    assert np.isnan(out[:, :13]).all() and np.isnan(out[:, 333:]).all()
    assert np.array_equal(out, want, equal_nan=True)
