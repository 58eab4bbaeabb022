"""Converted checkpoints run on the GPU engine as on the reference engine.

Tiny llama / qwen2 / qwen3moe Hugging Face checkpoints, converted to the Q4_K_M mix by
sardyne_b200.convert, are loaded through the reference's unmodified runtime on this library and on
the reference library (oracle/_ref, scalar kernels). The prompt's logits must agree within the
engine tests' tolerance, and 16 greedy tokens must be identical. The qwen2 checkpoint carries a
tokenizer.json, and its prompt is text encoded by the reference's tokenizer read from the
converted file.
"""
import numpy as np
import pytest

import oracle
import refruntime as rt
from sardyne_b200 import convert
from test_convert import checkpoint, write_tokenizer

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not (oracle.ref_available() and rt.available()),
                                                  reason="needs the reference library and its Python package")]

TOKENS = [3, 14, 15, 9, 26, 5, 35, 8, 2, 7, 1, 60]


@pytest.fixture(scope="module")
def ref_lib():
    lib = oracle.ref()
    lib.op_set_simd(0)
    yield oracle.REF_LIB
    lib.op_set_simd(1)


@pytest.mark.parametrize("arch,tied", [("llama", True), ("qwen2", False), ("qwen3moe", False)])
def test_converted_model_matches_reference_engine(tmp_path, ref_lib, arch, tied):
    ck = checkpoint(tmp_path, arch, tied)
    tokens = TOKENS
    if arch == "qwen2":
        rt.modules()
        write_tokenizer(ck, "qwen2", convert.QWEN2_SPLIT)
    path = convert.convert(ck, tmp_path / "m.gguf", "q4_k_m")
    if arch == "qwen2":
        from sardyne.tokenizer.bpe import BPETokenizer  # the reference's, reading the converted file
        tokens = BPETokenizer.load(model=path).encode("abc ab a12 cab<|endoftext|>abc x a1")
        assert len(tokens) >= 8
    want = rt.Context(rt.model(path, ref_lib), max_seq=48, n_batch=len(tokens), logits_all=True).eval(tokens)
    got = rt.Context(rt.model(path), max_seq=48, n_batch=len(tokens), logits_all=True).eval(tokens)
    tol = 1e-3 * max(1.0, float(np.abs(want).max()))
    assert np.abs(got - want).max() <= tol, (float(np.abs(got - want).max()), tol)
    assert (got.argmax(-1) == want.argmax(-1)).all()
    a = rt.generate(rt.Context(rt.model(path, ref_lib), max_seq=48), tokens[:4], 16)
    b = rt.generate(rt.Context(rt.model(path), max_seq=48), tokens[:4], 16)
    assert len(a) == 16 and a == b
