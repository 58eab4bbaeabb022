"""Generate the golden vectors that pin the CPU oracle (run where the reference is mounted).

    python tests/golden/make_golden.py <reference source tree>   (or SARDYNE_REFERENCE=<tree>)

Everything stored here is produced by the reference itself:
  * block bytes from the reference's own fixture generator ``random_blocks``
    (reference tests/test_quant.py:24-36);
  * outputs of the reference C library (built from its sources by oracle/Makefile) through the
    reference's own ctypes layer ``sardyne.capi`` (SARDYNE_LIB points at the built library):
    ``op_row_to_f32`` (dequant), ``op_quantize_rows`` (Q8_0 / Q8_K), ``op_vec_dot_q`` and
    ``op_matmul_q_rows`` with both the scalar and the AVX2 kernels;
  * the reference NumPy twin ``sardyne.quant`` (dequantize / quantize) for the same inputs.
The cases mirror the reference tests: tests/test_quant.py:132-205.
"""
import os
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = pathlib.Path(sys.argv[1] if len(sys.argv) > 1 else os.environ["SARDYNE_REFERENCE"])
os.environ["SARDYNE_LIB"] = str(REPO / "oracle" / "_ref" / "libsardyne_ref.so")
sys.path.insert(0, str(REF))
sys.path.insert(0, str(REF / "tests"))

from sardyne import capi, quant  # noqa: E402  (the reference's modules)
from sardyne.loader.gguf import GGML_TYPE_ID  # noqa: E402
from test_quant import random_blocks  # noqa: E402  (the reference's fixture generator)

KINDS = ["Q8_0", "Q4_0", "Q5_0", "Q4_K", "Q6_K"]


def ptr(a):
    return a.ctypes.data


def main():
    lib = capi.lib()
    out = {}

    # random_blocks itself (so the oracle's restatement can be pinned byte for byte)
    for kind in KINDS:
        out[f"blocks_{kind}_s0"] = random_blocks(kind, 16, seed=0)

    # dequant (test_quant.py:132-139): C and NumPy must agree bit for bit
    n = 2048
    for kind in KINDS:
        row = random_blocks(kind, n // quant.QK[kind], seed=4).reshape(-1)
        got = np.empty(n, np.float32)
        lib.op_row_to_f32(ptr(row), GGML_TYPE_ID[kind], ptr(got), n)
        assert np.array_equal(got, quant.dequantize(row, kind, (n,)))
        out[f"deq_{kind}_w"], out[f"deq_{kind}_y"] = row, got

    # activation quantization (test_quant.py:141-151) plus extra edge blocks
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((3, 512)) * np.array([[1e-3], [1.0], [300.0]])).astype(np.float32)
    x[1, :256] = 0
    x[2, 7] = 1e4
    edge = np.zeros((4, 512), np.float32)
    edge[0, :] = 1e-30                                    # tiny, nonzero (subnormal-ish products)
    edge[1, 3], edge[1, 9] = -2.5, 2.5                    # tie on |max|: first index (negative) wins
    edge[2, :] = np.float32(0.5) + np.arange(512, dtype=np.float32) / 512  # .5 ties after scaling
    edge[3, 0:256] = rng.standard_normal(256).astype(np.float32) * 1e4
    edge[3, 256:] = -np.float32(3.0)
    x = np.concatenate([x, edge])
    out["act_x"] = x
    for vt in ("Q8_0", "Q8_K"):
        q = np.zeros(lib.op_row_size(GGML_TYPE_ID[vt], x.shape[1]) * x.shape[0], np.uint8)
        lib.op_quantize_rows(GGML_TYPE_ID[vt], ptr(x), ptr(q), x.shape[1], 0, x.shape[0])
        assert q.tobytes() == quant.quantize(x, vt)
        out[f"act_{vt}"] = q

    # vec_dot (test_quant.py:154-185): scalar and AVX2 results from the reference C kernels
    n = 1024
    for kind in KINDS:
        w = random_blocks(kind, n // quant.QK[kind], seed=6).reshape(-1)
        xv = np.random.default_rng(7).standard_normal(n).astype(np.float32)
        xq = np.frombuffer(quant.quantize(xv, quant.VEC_DOT_TYPE[kind]), np.uint8).copy()
        res = []
        for simd in (0, 1):
            lib.op_set_simd(simd)
            res.append(lib.op_vec_dot_q(GGML_TYPE_ID[kind], ptr(w), ptr(xq), n))
        lib.op_set_simd(1)
        out[f"dot_{kind}_w"], out[f"dot_{kind}_xq"] = w, xq
        out[f"dot_{kind}_scalar_avx2"] = np.array(res, np.float32)

    # matmul_q_rows (test_quant.py:188-205) and a larger multi-token case
    for (n_in, n_out, n_tok, seed, tag) in [(512, 13, 3, 10, "small"), (2048, 40, 9, 20, "big")]:
        for kind in KINDS:
            w = random_blocks(kind, n_out * n_in // quant.QK[kind], seed=seed).reshape(n_out, -1)
            xv = np.random.default_rng(seed + 1).standard_normal((n_tok, n_in)).astype(np.float32)
            vt = quant.VEC_DOT_TYPE[kind]
            xq = np.frombuffer(quant.quantize(xv, vt), np.uint8).copy()
            res = {}
            for simd in (0, 1):
                lib.op_set_simd(simd)
                o = np.full((n_tok, n_out), np.nan, np.float32)
                lib.op_matmul_q_rows(ptr(o), ptr(xq), ptr(w), GGML_TYPE_ID[kind], n_tok, n_in, n_out, 0, n_out)
                res[simd] = o
            lib.op_set_simd(1)
            out[f"mm_{tag}_{kind}_w"], out[f"mm_{tag}_{kind}_xq"] = w, xq
            out[f"mm_{tag}_{kind}_scalar"], out[f"mm_{tag}_{kind}_avx2"] = res[0], res[1]
            out[f"mm_{tag}_{kind}_shape"] = np.array([n_in, n_out, n_tok], np.int64)

    # f32 -> f16 special values (test_quant.py:119-128): the reference C result
    v = np.array([65504, 65519, 65520, 7e4, 6e-8, 3e-8, 2.98e-8, 0, -0.0, 5.96e-8, np.inf, -np.inf,
                  1.0009765625, 1.00048828125, 1.000732421875, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26,
                  -6.1e-5, 6.097e-5, 0.1, 1e-7], np.float32)
    out["f16_in"] = v
    out["f16_out"] = np.array([lib.op_f32_to_f16(float(a)) for a in v], np.uint16)

    np.savez_compressed(HERE / "quant_golden.npz", **out)
    print(f"wrote {HERE / 'quant_golden.npz'} ({len(out)} arrays)")


if __name__ == "__main__":
    main()
