"""sardyne_b200 — B200-native drop-in for Sardyne's quantized-weight hot path.

The product is libsardyne.so (sardyne_b200/csrc, built by sardyne_b200/build.py), exporting the
reference's C-ABI (include/sardyne_b200.h). This package holds the build script, a ctypes
binding with the reference's symbol table (capi), a model-level wrapper mirroring the
reference's runtime (runtime), and the GGUF writer and K-quant quantizer used to make
synthetic models (gguf_writer, kquant).
"""
from . import capi  # noqa: F401

__all__ = ["capi"]
