"""CPU oracle for the quantized-weight hot path — TEST INFRASTRUCTURE, not the product.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs import this
package, and only as the checker or the timed CPU baseline. The product (sardyne_b200/) never
imports it.

Two checkers live here:
  * ``qref`` — liboracle.so, a plain-C restatement of the reference's scalar kernels
    (reference csrc/quant.c:13-235, csrc/ops.c:15-62,293-309), built by oracle/Makefile.
    Pinned against golden vectors made by the reference itself (tests/golden/).
  * ``ref`` — oracle/_ref/libsardyne_ref.so, the reference library compiled from its own
    sources by oracle/Makefile (present wherever it was built; it travels as a built file).
"""
import ctypes
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "liboracle.so"
REF_LIB = HERE / "_ref" / "libsardyne_ref.so"

# ggml type ids (reference csrc/ops.h:21-22)
F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q6_K, Q8_K, BF16 = 0, 1, 2, 6, 8, 12, 14, 15, 30
TYPE_ID = {"F32": F32, "F16": F16, "Q4_0": Q4_0, "Q5_0": Q5_0, "Q8_0": Q8_0, "Q4_K": Q4_K, "Q6_K": Q6_K,
           "Q8_K": Q8_K, "BF16": BF16}
QK = {"Q8_0": 32, "Q4_0": 32, "Q5_0": 32, "Q4_K": 256, "Q6_K": 256, "Q8_K": 256}
BLOCK_BYTES = {"Q8_0": 34, "Q4_0": 18, "Q5_0": 22, "Q4_K": 144, "Q6_K": 210, "Q8_K": 292}
VEC_DOT_TYPE = {"Q8_0": "Q8_0", "Q4_0": "Q8_0", "Q5_0": "Q8_0", "Q4_K": "Q8_K", "Q6_K": "Q8_K"}
WEIGHT_TYPES = ["Q8_0", "Q4_0", "Q5_0", "Q4_K", "Q6_K"]

_vp, _i = ctypes.c_void_p, ctypes.c_int
_oracle = None


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def qref() -> ctypes.CDLL:
    """The C restatement (oracle/qref.c)."""
    global _oracle
    if _oracle is None:
        if not ORACLE_LIB.exists():
            raise OSError(f"{ORACLE_LIB} missing: run `make -C oracle`")
        lib = ctypes.CDLL(str(ORACLE_LIB))
        lib.oq_f16_to_f32.restype, lib.oq_f16_to_f32.argtypes = ctypes.c_float, [ctypes.c_uint16]
        lib.oq_f32_to_f16.restype, lib.oq_f32_to_f16.argtypes = ctypes.c_uint16, [ctypes.c_float]
        lib.oq_dequant_row.restype, lib.oq_dequant_row.argtypes = None, [_i, _vp, _vp, _i]
        lib.oq_quantize_rows.restype, lib.oq_quantize_rows.argtypes = None, [_i, _vp, _vp, _i, _i]
        lib.oq_vec_dot.restype, lib.oq_vec_dot.argtypes = ctypes.c_float, [_i, _vp, _vp, _i]
        lib.oq_matmul_q_rows.restype = None
        lib.oq_matmul_q_rows.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i]
        lib.oq_row_bytes.restype, lib.oq_row_bytes.argtypes = ctypes.c_size_t, [_i, _i]
        lib.oq_expf_n.restype, lib.oq_expf_n.argtypes = None, [_vp, _vp, ctypes.c_size_t]
        _oracle = lib
    return _oracle


def expf(x) -> np.ndarray:
    """libm's expf element by element: the exp the reference's fp32 code calls."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    qref().oq_expf_n(_ptr(x), _ptr(y), x.size)
    return y


def row_bytes(kind: str, n: int) -> int:
    return n // QK[kind] * BLOCK_BYTES[kind]


def dequant(raw: np.ndarray, kind: str, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8).reshape(-1)
    rows = raw.size // row_bytes(kind, n)
    out = np.empty((rows, n), np.float32)
    rb = row_bytes(kind, n)
    for r in range(rows):
        qref().oq_dequant_row(TYPE_ID[kind], _ptr(raw) + r * rb, _ptr(out) + r * n * 4, n)
    return out


def quantize(x: np.ndarray, vkind: str) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    x2 = x.reshape(-1, x.shape[-1])
    out = np.zeros(row_bytes(vkind, x2.shape[1]) * x2.shape[0], np.uint8)
    qref().oq_quantize_rows(TYPE_ID[vkind], _ptr(x2), _ptr(out), x2.shape[1], x2.shape[0])
    return out


def vec_dot(w: np.ndarray, kind: str, xq: np.ndarray, n: int) -> float:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    return qref().oq_vec_dot(TYPE_ID[kind], _ptr(w), _ptr(xq), n)


def matmul_q(w: np.ndarray, kind: str, xq: np.ndarray, n_tok: int, n_in: int, n_out: int,
             row0: int = 0, row1: int | None = None, out: np.ndarray | None = None) -> np.ndarray:
    row1 = n_out if row1 is None else row1
    w = np.ascontiguousarray(w, dtype=np.uint8)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    if out is None:
        out = np.zeros((n_tok, n_out), np.float32)
    qref().oq_matmul_q_rows(_ptr(out), _ptr(xq), _ptr(w), TYPE_ID[kind], n_tok, n_in, n_out, row0, row1)
    return out


def random_blocks(kind: str, n_blocks: int, seed: int = 0) -> np.ndarray:
    """Random block bytes with sane fp16 scales: the reference's own K-quant fixture generator
    (reference tests/test_quant.py:24-36), restated so it runs where the reference is absent.
    tests/test_oracle_golden.py checks its bytes against the reference's output."""
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, (n_blocks, BLOCK_BYTES[kind]), dtype=np.uint8)

    def scale():
        return rng.uniform(1e-4, 1e-2, n_blocks).astype(np.float16).view(np.uint8).reshape(-1, 2)

    if kind in ("Q8_0", "Q4_0", "Q5_0"):
        b[:, 0:2] = scale()
    elif kind == "Q4_K":
        b[:, 0:2] = scale()
        b[:, 2:4] = scale()
    elif kind == "Q6_K":
        b[:, 208:210] = scale()
        b[:, 192:208] = rng.integers(-60, 60, (n_blocks, 16)).astype(np.int8).view(np.uint8)
    return b


def special_rows(n: int) -> np.ndarray:
    """Activation rows of special values (n a multiple of 512): signed zeros, blocks whose largest
    magnitude is so small (subnormal, below ~3.7e-37) that the quantizers' inverse scale overflows
    to infinity, values near the float maximum, a negative maximum, and normal blocks beside tiny
    ones in the same row. The reference's quantizers give defined bytes for all of them."""
    rows = [np.full(n, -0.0, np.float32)]
    r = np.zeros(n, np.float32); r[5], r[7], r[40] = 1e-40, -3e-41, 2e-45; rows.append(r)
    r = np.full(n, 1.5e-39, np.float32); r[::3] *= -1; rows.append(r)
    r = np.full(n, -2e-38, np.float32); r[1::2] = 1e-38; rows.append(r)  # negative maximum, tiny
    r = np.zeros(n, np.float32); r[1], r[2], r[3] = 3.0e38, -1e-30, 1.0; rows.append(r)
    r = np.linspace(-2.0, 1.0, n).astype(np.float32); rows.append(r)
    r = np.random.default_rng(0).standard_normal(n).astype(np.float32)
    r[256:512] *= 1e-38; r[300] = -4e-39; rows.append(r)  # a normal block, then tiny ones
    return np.ascontiguousarray(np.stack(rows))


# ---------------------------------------------------------------- the reference library itself

def ref_available() -> bool:
    return REF_LIB.exists()


_ref = None


def ref() -> ctypes.CDLL:
    """The reference libsardyne built from its own sources (oracle/Makefile), bound with the
    signatures of the reference's ctypes layer (reference sardyne/capi.py:33-102)."""
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise OSError(f"{REF_LIB} missing: run `make -C oracle` where the reference sources exist")
        lib = ctypes.CDLL(str(REF_LIB))
        _i32, _fp = ctypes.c_int32, ctypes.POINTER(ctypes.c_float)
        sig = {
            "op_simd": (_i, []), "op_set_simd": (_i, [_i]),
            "op_row_to_f32": (None, [_vp, _i, _vp, ctypes.c_size_t]),
            "op_quantize_rows": (None, [_i, _vp, _vp, _i, _i, _i]),
            "op_matmul_q_rows": (None, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i]),
            "op_vec_dot_q": (ctypes.c_float, [_i, _vp, _vp, _i]),
            "op_matmul": (None, [_vp, _vp, _vp, _i, _i, _i, _i]),
            "op_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
            "op_attention": (None, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
            "engine_model_load": (_vp, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]),
            "engine_model_free": (None, [_vp]),
            "engine_ctx_new": (_vp, [_vp, _i32, _i32, _i32, _i32, ctypes.c_char_p, ctypes.c_size_t]),
            "engine_ctx_free": (None, [_vp]),
            "engine_eval": (_i, [_vp, ctypes.POINTER(_i32), _i32]),
            "engine_logits": (_fp, [_vp]),
            "engine_n_logits": (_i32, [_vp]),
            "engine_n_past": (_i32, [_vp]),
            "engine_last_error": (ctypes.c_char_p, [_vp]),
            "engine_model_get_info": (None, [_vp, _vp]),
            "engine_ctx_n_threads": (_i32, [_vp]),
            "engine_reset": (None, [_vp]),
            "engine_truncate": (_i, [_vp, _i32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype, fn.argtypes = res, args
        _ref = lib
    return _ref
