"""sdy_qmatvec_f32_noalloc: the entry point for callers that cannot allocate device memory where
they call it (a host framework that accounts for all device memory through its own pool, or a
serving loop that keeps cudaMalloc/cudaFree out of its steady state). Its output must equal the
allocating entry points' (op_matmul through host buffers, and sdy_quantize_rows_dev +
sdy_qmatvec_dev), bit for bit as every product test here, on consecutive calls that reuse its one
internal scratch array, on both the CUDA-core matvec (under 32 tokens) and the tensor-core route
(32 tokens and more for Q4_K/Q6_K).

The file name sorts last so that a run stopping at the first failure has run everything else.
"""
import ctypes

import numpy as np
import pytest

import oracle
from sardyne_b200 import capi

pytestmark = pytest.mark.gpu


def vp(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("kind", ["Q4_K", "Q6_K", "Q8_0", "Q5_0"])
def test_noalloc_matches_allocating_entry_points(kind):
    import torch

    lib = capi.lib()
    lib.sdy_clear_error()
    n_in, n_out = 2048, 1000
    w = oracle.random_blocks(kind, n_out * n_in // oracle.QK[kind], seed=3)
    h = lib.sdy_qmat_upload(w.ctypes.data, oracle.TYPE_ID[kind], n_out, n_in)
    assert h, capi.last_error()
    try:
        vt = oracle.TYPE_ID[oracle.VEC_DOT_TYPE[kind]]
        rng = np.random.default_rng(7)
        # two calls in a row with different data and token counts: the shared scratch keeps
        # the first call's contents when the second starts
        calls = [(5, (0, n_out)), (2, (129, 871))]
        if kind in ("Q4_K", "Q6_K"):
            calls.append((40, (8, 1000)))  # 32 tokens and more: the tensor-core GEMM
        for n_tok, (r0, r1) in calls:
            x = rng.standard_normal((n_tok, n_in)).astype(np.float32)
            dx = torch.from_numpy(x).cuda()
            got = torch.full((n_tok, r1 - r0), float("nan"), device="cuda")
            assert lib.sdy_qmatvec_f32_noalloc(h, vp(dx), n_tok, vp(got), r1 - r0, r0, r1, None) == 0, \
                capi.last_error()
            xq = torch.empty(lib.sdy_xq_bytes(vt, n_in, n_tok), dtype=torch.uint8, device="cuda")
            dev = torch.full((n_tok, r1 - r0), float("nan"), device="cuda")
            assert lib.sdy_quantize_rows_dev(vt, vp(dx), n_tok, n_in, vp(xq), None) == 0
            assert lib.sdy_qmatvec_dev(h, vp(xq), n_tok, vp(dev), r1 - r0, r0, r1, None) == 0
            host = np.full((n_tok, n_out), np.nan, np.float32)
            lib.op_matmul(host.ctypes.data, x.ctypes.data, w.ctypes.data, oracle.TYPE_ID[kind], n_tok, n_in, n_out)
            torch.cuda.synchronize()
            capi.check()
            g = got.cpu().numpy()
            assert np.array_equal(g, dev.cpu().numpy())
            assert np.array_equal(g, host[:, r0:r1])
    finally:
        lib.sdy_qmat_free(h)


def test_noalloc_rejects_requests_beyond_its_scratch():
    """512 KiB of quantized activations: 26 tokens of 16384 elements fit, 27 do not."""
    import torch

    lib = capi.lib()
    n_in, n_out = 16384, 8
    w = oracle.random_blocks("Q4_K", n_out * n_in // 256, seed=4)
    h = lib.sdy_qmat_upload(w.ctypes.data, oracle.TYPE_ID["Q4_K"], n_out, n_in)
    assert h, capi.last_error()
    try:
        assert lib.sdy_xq_bytes(15, n_in, 26) <= 512 * 1024 < lib.sdy_xq_bytes(15, n_in, 27)
        x = torch.zeros((27, n_in), device="cuda")
        out = torch.zeros((27, n_out), device="cuda")
        assert lib.sdy_qmatvec_f32_noalloc(h, vp(x), 27, vp(out), n_out, 0, n_out, None) == -1
        assert b"scratch" in lib.sdy_last_error()
        lib.sdy_clear_error()
        assert lib.sdy_qmatvec_f32_noalloc(h, vp(x), 26, vp(out), n_out, 0, n_out, None) == 0, capi.last_error()
        torch.cuda.synchronize()
        assert not out[:26].any()  # zero activations give zero products
    finally:
        lib.sdy_qmat_free(h)
