"""The reference's own Python layer, unmodified, binds and drives this library (CPU part).

With SARDYNE_LIB naming the B200 build, the reference's sardyne.capi.lib() binds every name of its
signature table (it fails on a missing one, reference sardyne/capi.py:105-124) and its
sardyne.runtime.Model reports the library's load errors as the reference does
(sardyne/runtime.py:34-48). Header checks run before any GPU work, so a malformed model is refused
with the reference's message here; a valid one is refused on a machine without a GPU. The GPU
engine tests drive the same runtime end to end (tests/test_gpu_engine.py,
tests/test_gpu_baseline_shapes.py).
"""
import os
import pathlib
import subprocess
import sys

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


def _reference_tests():
    root = os.environ.get("SARDYNE_REFERENCE")
    return pathlib.Path(root) / "tests" if root else None


@pytest.mark.skipif(not (_reference_tests() and (_reference_tests() / "test_gguf.py").exists()),
                    reason="set SARDYNE_REFERENCE to the reference's source tree")
def test_reference_gguf_and_capi_tests_pass_on_this_library(tmp_path):
    """The reference's own tests/test_gguf.py and tests/test_capi.py, unmodified, with SARDYNE_LIB
    naming this build. Their C-reader cases go through this library's gguf_* functions: round trips,
    custom alignment, truncated, corrupted and bad-magic/version files, the rejection rules shared
    with the Python reader, the error messages and the binding's lifecycle. Excluded: test_capi's
    `add`, which computes on a GPU, and the cases that need downloaded models, which skip."""
    tests = _reference_tests()
    env = dict(os.environ, SARDYNE_LIB=str(rt.b200_lib()), PYTHONPATH=str(tests.parent), PYTHONDONTWRITEBYTECODE="1")
    r = subprocess.run([sys.executable, "-m", "pytest", str(tests / "test_gguf.py"), str(tests / "test_capi.py"),
                        "-k", "not add_matches", "-q", "-p", "no:cacheprovider"],
                       cwd=tmp_path, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and " failed" not in r.stdout, r.stdout[-2000:]
