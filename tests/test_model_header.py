"""Model header and tensor-name validation of engine_model_load, against the reference library.

Both libraries read the same malformed GGUFs; the B200 build must refuse each with the reference's
message (reference csrc/model_llama.c:225-319; its tests match these texts, e.g.
tests/test_runtime.py:379-399 and tests/test_moe.py:409-435). The checks run before any GPU work,
so this runs on the CPU. The one intended difference: the reference's rope-scaling message names a
roadmap phase, this build's says "non supportato"; both start with "rope scaling".
"""
import ctypes

import numpy as np
import pytest

import oracle
from sardyne_b200 import capi
from sardyne_b200.gguf_writer import F32, STRING, U32, GGUFWriter

pytestmark = pytest.mark.skipif(not (capi.available() and oracle.ref_available()),
                                reason="needs the built library and the reference library")

BASE = {"embedding_length": 32, "block_count": 2, "feed_forward_length": 64, "attention.head_count": 4,
        "attention.head_count_kv": 2, "context_length": 64, "attention.layer_norm_rms_epsilon": 1e-5,
        "rope.freq_base": 10000.0}
MOE = {"expert_count": 8, "expert_used_count": 2, "expert_feed_forward_length": 16}


def write(path, arch="llama", meta=None, drop=(), tensors=None, arch_value=None):
    w = GGUFWriter(path)
    w.add("general.architecture", arch if arch_value is None else arch_value)
    kv = dict(BASE, **(MOE if arch == "qwen3moe" else {}))
    kv.update(meta or {})
    for k, v in kv.items():
        if k in drop:
            continue
        if isinstance(v, str):
            w.add(f"{arch}.{k}", v, STRING)
        elif isinstance(v, float):
            w.add(f"{arch}.{k}", v, F32)
        else:
            w.add(f"{arch}.{k}", v, U32)
    for name in tensors if tensors is not None else ["token_embd.weight"]:
        w.add_tensor(name, np.zeros((8, 32), np.float32))
    return w.write()


def load_error(lib, path):
    lib.engine_model_load.restype = ctypes.c_void_p
    lib.engine_model_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]
    lib.engine_model_free.argtypes = [ctypes.c_void_p]
    err = ctypes.create_string_buffer(512)
    h = lib.engine_model_load(str(path).encode(), err, len(err))
    if h:
        lib.engine_model_free(h)
        return None
    return err.value.decode()


CASES = {
    "arch-missing": dict(arch_value=""),
    "arch-unknown": dict(arch="gpt2"),
    "rope-scaling": dict(meta={"rope.scaling.type": "linear"}),
    "rope-freqs-tensor": dict(tensors=["token_embd.weight", "rope_freqs.weight"]),
    "dim-missing": dict(drop=("embedding_length",)),
    "dim-zero": dict(meta={"embedding_length": 0}),
    "dim-huge": dict(meta={"embedding_length": (1 << 30) + 1}),
    "dim-string": dict(meta={"embedding_length": "32"}),
    "layers-missing": dict(drop=("block_count",)),
    "ffn-missing": dict(drop=("feed_forward_length",)),
    "heads-missing": dict(drop=("attention.head_count",)),
    "kv-heads-bad": dict(meta={"attention.head_count_kv": 3}),
    "key-length-zero-default": dict(meta={"attention.head_count": 64, "attention.head_count_kv": 64}),
    "value-length-differs": dict(meta={"attention.value_length": 16}),
    "value-length-invalid": dict(meta={"attention.value_length": 0}),
    "partial-rope": dict(meta={"rope.dimension_count": 4}),
    "odd-head-dim": dict(meta={"attention.key_length": 7, "attention.value_length": 7, "rope.dimension_count": 7}),
    "eps-missing": dict(drop=("attention.layer_norm_rms_epsilon",)),
    "eps-negative": dict(meta={"attention.layer_norm_rms_epsilon": -1.0}),
    "eps-integer": dict(meta={"attention.layer_norm_rms_epsilon": 3}),
    "theta-zero": dict(meta={"rope.freq_base": 0.0}),
    "context-zero": dict(meta={"context_length": 0}),
    "embedding-missing": dict(tensors=[]),
    "unknown-tensor": dict(tensors=["token_embd.weight", "blk.0.attn_qkv.weight"]),
    "layer-out-of-range": dict(tensors=["token_embd.weight", "blk.2.attn_q.weight"]),
    "layer-no-digits": dict(tensors=["token_embd.weight", "blk..attn_q.weight"]),
    "layer-no-dot": dict(tensors=["token_embd.weight", "blk.0attn_q.weight"]),
    "layer-huge-index": dict(tensors=["token_embd.weight", "blk.99999999999999999999.attn_q.weight"]),
    "moe-count-missing": dict(arch="qwen3moe", drop=("expert_count",)),
    "moe-used-missing": dict(arch="qwen3moe", drop=("expert_used_count",)),
    "moe-used-zero": dict(arch="qwen3moe", meta={"expert_used_count": 0}),
    "moe-used-over-count": dict(arch="qwen3moe", meta={"expert_used_count": 9}),
    "moe-ffn-zero-default": dict(arch="qwen3moe", meta={"feed_forward_length": 1}, drop=("expert_feed_forward_length",)),
    "moe-ffn-invalid": dict(arch="qwen3moe", meta={"expert_feed_forward_length": 0}),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_refused_like_the_reference(tmp_path, case):
    path = write(tmp_path / f"{case}.gguf", **CASES[case])
    want = load_error(oracle.ref(), path)
    got = load_error(capi.lib(), path)
    assert want, "the reference accepted this file"
    if case.startswith("rope"):
        assert got.startswith("rope scaling") and want.startswith("rope scaling"), (got, want)
    else:
        assert got == want


def test_leading_zero_layer_index_is_accepted(tmp_path):
    """'blk.01.' names layer 1 for both libraries: the header check passes (the reference then
    fails on the missing layer tensors; this build, on the CPU, too, or on the absent GPU)."""
    path = write(tmp_path / "z.gguf", tensors=["token_embd.weight", "blk.01.attn_q.weight"])
    for lib in (oracle.ref(), capi.lib()):
        assert "non supportato" not in load_error(lib, path)
