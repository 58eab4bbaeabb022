"""ctypes binding of libsardyne.so (the B200 build).

The symbol table is the reference's (sardyne/capi.py:33-102: same names, same argument and
return types) so that the reference's own Python layer binds this library unchanged with
SARDYNE_LIB pointing at it. ``lib()`` binds every name at load, as the reference does, so a
missing export fails loudly at load time. The B200 extensions (include/sardyne_b200.h, last
block) are bound on top.
"""
import ctypes
import os
import pathlib

import numpy as np

PKG = pathlib.Path(__file__).resolve().parent
DEFAULT_LIB = PKG / "lib" / "libsardyne.so"

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u64 = ctypes.c_uint64
_vp, _i32, _fp = ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_float)
_i, _sz = ctypes.c_int, ctypes.c_size_t


class GGUFTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("n_dims", ctypes.c_uint32), ("type", ctypes.c_uint32),
                ("ne", ctypes.c_uint64 * 4), ("offset", ctypes.c_uint64), ("nbytes", ctypes.c_uint64),
                ("data", ctypes.c_void_p)]


class GGUFKV(ctypes.Structure):
    _fields_ = [("key", ctypes.c_char_p), ("type", ctypes.c_uint32), ("arr_type", ctypes.c_uint32),
                ("n", ctypes.c_uint64), ("ptr", ctypes.c_void_p), ("str_pos", ctypes.c_void_p)]


class EngineModelInfo(ctypes.Structure):
    _fields_ = [(name, ctypes.c_int32) for name in
                ("n_vocab", "dim", "n_layer", "n_head", "n_kv_head", "head_dim", "ffn_dim", "max_pos")] + \
               [("norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float)] + \
               [(name, ctypes.c_int32) for name in ("rope_interleaved", "qkv_bias", "tied_embeddings", "qk_norm",
                                                    "n_expert", "n_expert_used", "ffn_exp_dim")]


# The reference's exported surface (sardyne/capi.py:33-102).
SIGNATURES = {
    "engine_version": (ctypes.c_char_p, []),
    "engine_add_f32": (None, [_f32p, _f32p, _f32p, _sz]),
    "gguf_open": (_vp, [ctypes.c_char_p, ctypes.c_char_p, _sz]),
    "gguf_close": (None, [_vp]),
    "gguf_version": (ctypes.c_uint32, [_vp]),
    "gguf_alignment": (ctypes.c_uint32, [_vp]),
    "gguf_data_offset": (_u64, [_vp]),
    "gguf_n_kv": (_u64, [_vp]),
    "gguf_n_tensors": (_u64, [_vp]),
    "gguf_get_kv": (ctypes.POINTER(GGUFKV), [_vp, _u64]),
    "gguf_find_kv": (ctypes.c_int64, [_vp, ctypes.c_char_p]),
    "gguf_get_tensor": (ctypes.POINTER(GGUFTensor), [_vp, _u64]),
    "gguf_find_tensor": (ctypes.c_int64, [_vp, ctypes.c_char_p]),
    "gguf_kv_get_u64": (_i, [_vp, ctypes.c_int64, ctypes.POINTER(_u64)]),
    "gguf_kv_get_f64": (_i, [_vp, ctypes.c_int64, ctypes.POINTER(ctypes.c_double)]),
    "gguf_kv_get_str": (_vp, [_vp, ctypes.c_int64, ctypes.POINTER(_u64)]),
    "gguf_kv_get_arr_str": (_vp, [_vp, ctypes.c_int64, _u64, ctypes.POINTER(_u64)]),
    "gguf_type_name": (ctypes.c_char_p, [ctypes.c_uint32]),
    "engine_model_load": (_vp, [ctypes.c_char_p, ctypes.c_char_p, _sz]),
    "engine_model_free": (None, [_vp]),
    "engine_model_get_info": (None, [_vp, ctypes.POINTER(EngineModelInfo)]),
    "engine_ctx_new": (_vp, [_vp, _i32, _i32, _i32, _i32, ctypes.c_char_p, _sz]),
    "engine_ctx_n_threads": (_i32, [_vp]),
    "engine_ctx_free": (None, [_vp]),
    "engine_eval": (_i, [_vp, ctypes.POINTER(_i32), _i32]),
    "engine_logits": (_fp, [_vp]),
    "engine_n_logits": (_i32, [_vp]),
    "engine_n_past": (_i32, [_vp]),
    "engine_reset": (None, [_vp]),
    "engine_truncate": (_i, [_vp, _i32]),
    "engine_last_error": (ctypes.c_char_p, [_vp]),
    "op_simd": (_i, []),
    "op_set_simd": (_i, [_i]),
    "op_f16_to_f32_n": (None, [_vp, _vp, _sz]),
    "op_matmul_rows": (None, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i]),
    "op_dot_f32": (ctypes.c_float, [_vp, _vp, _i]),
    "op_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
    "op_row_to_f32": (None, [_vp, _i, _vp, _sz]),
    "op_row_size": (_sz, [_i, _i]),
    "op_quantize_rows": (None, [_i, _vp, _vp, _i, _i, _i]),
    "op_matmul_q_rows": (None, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i]),
    "op_vec_dot_q": (ctypes.c_float, [_i, _vp, _vp, _i]),
    "op_axpy": (None, [_vp, ctypes.c_float, _vp, _i]),
    "op_matmul": (None, [_vp, _vp, _vp, _i, _i, _i, _i]),
    "op_rmsnorm": (None, [_vp, _vp, _vp, _i, ctypes.c_float]),
    "op_softmax": (None, [_vp, _i]),
    "op_silu_mul": (None, [_vp, _vp, _i]),
    "op_rope_table": (None, [_vp, _vp, _i, _i, ctypes.c_float]),
    "op_rope": (None, [_vp, _i, _i, _vp, _vp, _i]),
    "op_attention": (None, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]),
}

# B200 extensions (no reference counterpart).
EXTENSIONS = {
    "sdy_weights_register": (_i, [_vp, _i, ctypes.c_int64, _i32]),
    "sdy_weights_unregister": (_i, [_vp]),
    "sdy_last_error": (ctypes.c_char_p, []),
    "sdy_clear_error": (None, []),
    "sdy_kernel_launches": (_u64, []),
    "sdy_kernel_status": (ctypes.c_uint32, []),
    "sdy_kernel_clear_status": (None, []),
    "sdy_nccl_unique_id": (_i, [_vp]),
    "sdy_engine_set_shard": (_i, [ctypes.c_int32, ctypes.c_int32, _vp]),
    "sdy_engine_get_shard": (None, [ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]),
    "sdy_engine_eval_greedy": (_i, [_vp, ctypes.POINTER(_i32), _i32, ctypes.POINTER(_i32)]),
    "sdy_attention_split": (_i, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                 ctypes.POINTER(ctypes.c_int32)]),
    "sdy_engine_exchange": (_i, [_vp]),
    "sdy_shard_range": (None, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int64,
                               ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]),
    "sdy_qmat_upload": (_vp, [_vp, _i, ctypes.c_int64, _i32]),
    "sdy_qmat_free": (None, [_vp]),
    "sdy_qmat_bytes": (_sz, [_vp]),
    "sdy_xq_bytes": (_sz, [_i, _i, _i]),
    "sdy_quantize_rows_dev": (_i, [_i, _vp, _i, _i, _vp, _vp]),
    "sdy_qmatvec_dev": (_i, [_vp, _vp, _i, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp]),
    "sdy_qmatvec_batch_dev": (_i, [_i, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_vp), _vp]),
    "sdy_qmatvec_batch_f32_dev": (_i, [_i, ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_vp), _vp]),
    "sdy_qmatvec_batch_f32_gather_dev": (_i, [_i, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                              ctypes.POINTER(ctypes.c_int64), ctypes.c_int64, ctypes.POINTER(_vp),
                                              ctypes.c_int32, ctypes.c_int32, _vp]),
    "sdy_allgather_p2p_bytes": (_sz, [ctypes.c_int64, ctypes.c_int32]),
    "sdy_p2p_alloc": (_vp, [_sz]),
    "sdy_p2p_free": (None, [_vp]),
    "sdy_p2p_handle": (_i, [_vp, _vp]),
    "sdy_p2p_open": (_vp, [_vp]),
    "sdy_p2p_close": (_i, [_vp]),
    "sdy_allgather_p2p": (_i, [_vp, ctypes.c_int64, ctypes.POINTER(_vp), ctypes.c_int32, ctypes.c_int32, _vp]),
    "sdy_p2p_read": (_i, [_vp, _vp, _sz]),
    "sdy_p2p_status": (ctypes.c_uint32, []),
    "sdy_p2p_clear_status": (None, []),
    "sdy_qmatvec_f32_noalloc": (_i, [_vp, _vp, _i, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _vp]),
}

_lib = None


def lib_path() -> pathlib.Path:
    return pathlib.Path(os.environ.get("SARDYNE_B200_LIB", DEFAULT_LIB))


def available() -> bool:
    return lib_path().exists()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = lib_path()
        if not path.exists():
            raise OSError(f"{path} not found: build it with `python -m sardyne_b200.build`")
        handle = ctypes.CDLL(str(path))
        for name, (res, args) in {**SIGNATURES, **EXTENSIONS}.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def last_error() -> str:
    return lib().sdy_last_error().decode("utf-8", errors="replace")


def check():
    """Raise if the last library call on this thread recorded an error."""
    msg = last_error()
    if msg:
        lib().sdy_clear_error()
        raise RuntimeError(msg)
