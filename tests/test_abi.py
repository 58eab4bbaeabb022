"""The C-ABI library loads without a GPU and exports every symbol the header declares."""
import ctypes
import pathlib
import re

import pytest

from sardyne_b200 import capi

REPO = pathlib.Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "sardyne_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b([a-z][a-z0-9_]*)\s*\(", text)) - {"sizeof"})


def reference_capi_source():
    """The reference's sardyne/capi.py: from its pip install under baseline/_ref, or from the
    source tree named by SARDYNE_REFERENCE."""
    import os
    for root in (REPO / "baseline" / "_ref", pathlib.Path(os.environ.get("SARDYNE_REFERENCE", "-"))):
        if (root / "sardyne" / "capi.py").exists():
            return root / "sardyne" / "capi.py"
    return None


def test_library_exports_every_declared_function():
    lib = ctypes.CDLL(str(capi.lib_path()))
    names = declared_functions()
    assert len(names) >= 55
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing


def test_binding_covers_header_and_loads():
    lib = capi.lib()  # binds every name, like the reference's capi.lib()
    assert set(capi.SIGNATURES) | set(capi.EXTENSIONS) == set(declared_functions())
    assert lib.engine_version() == b"0.0.1"
    assert lib.op_row_size(12, 512) == 288 and lib.op_row_size(14, 256) == 210 and lib.op_row_size(8, 64) == 68


def test_reference_symbol_table_is_covered():
    """Every name the reference's ctypes layer binds at load (sardyne/capi.py:33-102)."""
    ref = reference_capi_source()
    if ref is None:
        pytest.skip("the reference's Python package is not installed here")
    names = set(re.findall(r'"((?:engine|gguf|op)_[a-z0-9_]+)":', ref.read_text()))
    assert names and names <= set(capi.SIGNATURES)


def test_grouped_and_exchange_entry_points_reject_bad_arguments():
    """Argument checks of the grouped products, the fused gather and the exchanges return -1 with a
    message before any CUDA call (so they run without a GPU)."""
    lib = capi.lib()
    vp = ctypes.c_void_p
    none = (vp * 1)()
    for n in (0, 9):
        assert lib.sdy_qmatvec_batch_f32_dev(n, none, none, none, None) == -1
        assert "1..8 products" in capi.last_error()
        assert lib.sdy_qmatvec_batch_dev(n, none, none, none, None) == -1
    offs = (ctypes.c_int64 * 1)(0)
    bases = (vp * 9)()
    for count, rank, world in ((16, 0, 9), (16, 2, 2), (0, 0, 2), (16, -1, 2)):
        assert lib.sdy_qmatvec_batch_f32_gather_dev(1, none, none, offs, count, bases, rank, world, None) == -1
        assert "bad arguments" in capi.last_error()
    assert lib.sdy_qmatvec_batch_f32_gather_dev(1, (vp * 1)(1), (vp * 1)(16), offs, 16, bases, 0, 2, None) == -1
    assert "buffer of rank 0 missing" in capi.last_error()
    assert lib.sdy_allgather_p2p_bytes(100, 9) == 0 and lib.sdy_allgather_p2p_bytes(100, 0) == 0
    assert lib.sdy_allgather_p2p_bytes(100, 2) >= 2 * 100 * 4
    assert lib.sdy_allgather_p2p(None, 16, bases, 0, 2, None) == -1
    assert lib.sdy_engine_exchange(None) == -1
    lib.sdy_clear_error()


def test_host_side_entry_points_equal_the_reference_library():
    """The entry points that need no GPU (row sizes of every type id and length, the kernel-set
    switch) answer as the reference library built from its sources (csrc/ops.c:211-255,189-209)."""
    import oracle
    if not oracle.ref_available():
        pytest.skip("reference library not built")
    ours, ref = ctypes.CDLL(str(capi.lib_path())), oracle.ref()
    for lib in (ours, ref):
        lib.op_row_size.restype = ctypes.c_size_t
        lib.op_row_size.argtypes = [ctypes.c_int, ctypes.c_int]
    for t in range(-2, 45):
        for n in (0, 1, 31, 32, 33, 255, 256, 512, 2048, 11008):
            assert ours.op_row_size(t, n) == ref.op_row_size(t, n), (t, n)
    try:
        for enable in (0, 1, 0):
            assert ours.op_set_simd(enable) == ref.op_set_simd(enable)
            assert ours.op_simd() == ref.op_simd()
    finally:
        ours.op_set_simd(1)
        ref.op_set_simd(1)
