"""The reference's own Python layer, unmodified, binds and drives this library (CPU part).

With SARDYNE_LIB naming the B200 build, the reference's sardyne.capi.lib() binds every name of its
signature table (it fails on a missing one, reference sardyne/capi.py:105-124) and its
sardyne.runtime.Model reports the library's load errors as the reference does
(sardyne/runtime.py:34-48). Header checks run before any GPU work, so a malformed model is refused
with the reference's message here; a valid one is refused on a machine without a GPU. The GPU
engine tests drive the same runtime end to end (tests/test_gpu_engine.py,
tests/test_gpu_baseline_shapes.py).
"""
import numpy as np
import pytest

import refruntime as rt
from sardyne_b200 import capi, synth
from sardyne_b200.gguf_writer import GGUFWriter

pytestmark = pytest.mark.skipif(not (rt.available() and capi.available()),
                                reason="needs the reference's Python package and the built library")


def test_reference_capi_binds_every_symbol(monkeypatch):
    ref_capi, _ = rt.modules()
    monkeypatch.setenv("SARDYNE_LIB", str(rt.b200_lib()))
    monkeypatch.setattr(ref_capi, "_lib", None)
    lib = ref_capi.lib()
    assert ref_capi.version() == "0.0.1"
    assert set(ref_capi._SIGNATURES) <= set(capi.SIGNATURES)
    for name in ref_capi._SIGNATURES:
        assert getattr(lib, name).restype == ref_capi._SIGNATURES[name][0]
    assert lib.op_row_size(12, 512) == 288
    monkeypatch.setattr(ref_capi, "_lib", None)


def test_reference_runtime_reports_load_errors(tmp_path):
    with pytest.raises(ValueError, match="impossibile aprire"):
        rt.model(tmp_path / "missing.gguf")
    bad = GGUFWriter(tmp_path / "bad.gguf")
    bad.add("general.architecture", "qwen3moe")
    for k, v in [("embedding_length", 32), ("block_count", 1), ("feed_forward_length", 64),
                 ("attention.head_count", 2), ("expert_count", 4), ("expert_used_count", 5)]:
        bad.add(f"qwen3moe.{k}", v)
    bad.add_tensor("token_embd.weight", np.zeros((8, 32), np.float32))
    with pytest.raises(ValueError, match="expert_used_count=5 oltre expert_count=4"):
        rt.model(bad.write())


def test_reference_runtime_on_a_valid_model(tmp_path):
    """A valid model loads on a GPU box; without a GPU the runtime raises the library's message."""
    import torch
    path = synth.write_model(tmp_path / "m.gguf", synth.Spec())
    if torch.cuda.is_available():
        m = rt.model(path)
        assert m.info.n_vocab == 64 and m.info.dim == 64
    else:
        with pytest.raises(ValueError, match="GPU"):
            rt.model(path)
