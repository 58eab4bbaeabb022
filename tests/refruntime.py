"""The reference's own Python layer (sardyne.capi, sardyne.runtime), unmodified, for the tests.

The engine tests drive BOTH libraries through it: the B200 build (the drop-in under test) and the
reference's C library compiled from its sources (oracle/_ref, the checker). That the reference's
runtime runs this build unchanged is the drop-in claim itself (reference sardyne/capi.py:105-124,
sardyne/runtime.py:34-140).

The package comes from its pip install under baseline/_ref (it travels with the repository
snapshot), or from the source tree named by SARDYNE_REFERENCE. The reference's capi binds the
library named by SARDYNE_LIB once and caches it; `model()` points it at the requested library just
for the Model it creates (a Model, and every Context made from it, keeps its own library handle).
"""
import os
import pathlib
import sys

import pytest

REPO = pathlib.Path(__file__).resolve().parent.parent


def _roots():
    yield REPO / "baseline" / "_ref"
    if os.environ.get("SARDYNE_REFERENCE"):
        yield pathlib.Path(os.environ["SARDYNE_REFERENCE"])


def available() -> bool:
    return any((r / "sardyne" / "runtime.py").exists() for r in _roots())


def modules():
    """(capi, runtime) of the reference package; the test skips when it is not installed."""
    for root in _roots():
        if (root / "sardyne" / "runtime.py").exists():
            if str(root) not in sys.path:
                sys.path.insert(0, str(root))
            break
    else:
        pytest.skip("the reference's Python package is not installed (pip install --target baseline/_ref)")
    from sardyne import capi, runtime  # the reference's modules
    return capi, runtime


def b200_lib() -> pathlib.Path:
    from sardyne_b200 import capi
    return capi.lib_path()


def ref_lib() -> pathlib.Path:
    import oracle
    return oracle.REF_LIB


def model(path, lib_path=None):
    """runtime.Model(path) of the reference's runtime on `lib_path` (default: the B200 build)."""
    capi, runtime = modules()
    lib_path = pathlib.Path(lib_path or b200_lib())
    saved = os.environ.get("SARDYNE_LIB")
    capi._lib = None  # capi caches the library it bound first; bind this one for this Model
    os.environ["SARDYNE_LIB"] = str(lib_path)
    try:
        return runtime.Model(path)
    finally:
        capi._lib = None
        if saved is None:
            os.environ.pop("SARDYNE_LIB", None)
        else:
            os.environ["SARDYNE_LIB"] = saved


def Context(*args, **kwargs):
    return modules()[1].Context(*args, **kwargs)


def generate(*args, **kwargs):
    return modules()[1].generate(*args, **kwargs)
