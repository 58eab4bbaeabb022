"""Minimal GGUF v3 writer for synthetic models (metadata, float and pre-quantized tensors).

Layout (GGUF v3, little-endian): "GGUF", u32 version, u64 n_tensors, u64 n_kv; the key/value
pairs (string key, u32 value type, value); the tensor infos (string name, u32 n_dims, u64 ne[],
u32 ggml type, u64 offset); zero padding to the alignment; then each tensor's bytes at its
aligned offset. The file is written to a temporary name and renamed, so a reader that already
mapped an older file keeps seeing it intact.
"""
import os
import pathlib
import struct

import numpy as np

# value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
GGML_TYPES = {"F32": 0, "F16": 1, "Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q8_0": 8, "Q4_K": 12, "Q6_K": 14, "BF16": 30}
_BLOCK = {"F32": (1, 4), "F16": (1, 2), "BF16": (1, 2), "Q4_0": (32, 18), "Q4_1": (32, 20), "Q5_0": (32, 22),
          "Q8_0": (32, 34), "Q4_K": (256, 144), "Q6_K": (256, 210)}
_SCALAR_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
               U64: "<Q", I64: "<q", F64: "<d"}


def _str(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round to nearest even bf16 bit patterns (uint16)."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounded = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    nan = np.isnan(np.asarray(x, np.float32))
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


DEFAULT_ALIGNMENT = 32


def _check_name(what: str, name: str) -> None:
    """Keys and tensor names: non-empty UTF-8 without NUL (readers refuse anything else)."""
    if not isinstance(name, str) or not name or "\0" in name:
        raise ValueError(f"{what} {name!r} is not a non-empty string without NUL")
    name.encode("utf-8")  # lone surrogates raise UnicodeEncodeError, a ValueError


class GGUFWriter:
    def __init__(self, path, alignment: int = DEFAULT_ALIGNMENT):
        if not (isinstance(alignment, int) and 0 < alignment <= 1 << 16 and alignment & (alignment - 1) == 0):
            raise ValueError(f"alignment {alignment} is not a power of two up to 65536")
        self.path = pathlib.Path(path)
        self.alignment = alignment
        self.kv = []        # (key, type, payload bytes)
        self.tensors = []   # (name, ne, type name, bytes)
        self._keys, self._names = set(), set()
        if alignment != DEFAULT_ALIGNMENT:
            self.add("general.alignment", alignment, U32)

    def add(self, key: str, value, vtype: int | None = None, arr_type: int | None = None):
        _check_name("key", key)
        if key in self._keys:
            raise ValueError(f"key {key!r} added twice")
        if isinstance(value, np.generic):
            value = value.item()  # NumPy scalars as the Python value
        if vtype is None:
            if isinstance(value, bool):
                vtype = BOOL
            elif isinstance(value, int):
                vtype = U32 if 0 <= value < 2 ** 32 else I64
            elif isinstance(value, float):
                vtype = F32
            elif isinstance(value, str):
                vtype = STRING
            elif isinstance(value, (list, tuple)):
                vtype = ARRAY
            else:
                raise TypeError(f"{key}: unsupported value {type(value)}")
        if vtype == STRING:
            if not isinstance(value, str):
                raise TypeError(f"{key}: STRING needs a str")
            payload = _str(value)
        elif vtype == ARRAY:
            value = [v.item() if isinstance(v, np.generic) else v for v in value]
            kinds = {type(v) for v in value}
            if any(isinstance(v, (list, tuple, np.ndarray)) for v in value):
                raise TypeError(f"{key}: arrays of arrays are not supported")
            if len(kinds) > 1 and not kinds <= {int, float}:
                raise TypeError(f"{key}: array elements of different types {sorted(k.__name__ for k in kinds)}")
            if arr_type is None:
                if kinds == {str}:
                    arr_type = STRING
                elif kinds == {bool}:
                    arr_type = BOOL
                elif float in kinds:
                    arr_type = F32
                else:  # integers: int32 when every value fits, else the 64-bit type that holds them
                    lo, hi = (min(value), max(value)) if value else (0, 0)
                    arr_type = I32 if -2 ** 31 <= lo and hi < 2 ** 31 else U64 if lo >= 0 else I64
            try:
                body = b"".join(_str(v) for v in value) if arr_type == STRING else \
                    b"".join(struct.pack(_SCALAR_FMT[arr_type], v) for v in value)
            except struct.error as e:
                raise ValueError(f"{key}: {e}") from None
            payload = struct.pack("<IQ", arr_type, len(value)) + body
        else:
            if vtype not in _SCALAR_FMT:
                raise ValueError(f"{key}: unknown value type {vtype}")
            try:
                payload = struct.pack(_SCALAR_FMT[vtype], value)
            except struct.error as e:  # out of the type's range, or not a number
                raise ValueError(f"{key}: {value!r} does not fit value type {vtype} ({e})") from None
        self._keys.add(key)
        self.kv.append((key, vtype, payload))

    def add_tensor(self, name: str, data: np.ndarray, kind: str = "F32"):
        """Float tensor; data shape [..., n_in] (row-major, as PyTorch): ne = reversed shape."""
        data = np.asarray(data)
        if kind == "F32":
            raw = np.ascontiguousarray(data, np.float32).tobytes()
        elif kind == "F16":
            raw = np.ascontiguousarray(data, np.float16).tobytes()
        elif kind == "BF16":
            raw = (data if data.dtype == np.uint16 else f32_to_bf16(data)).tobytes()
        else:
            raise ValueError(f"{kind}: use add_raw_tensor for quantized data")
        self._tensor(name, tuple(reversed(data.shape)), kind, raw)

    def add_raw_tensor(self, name: str, ne, kind: str, raw: bytes):
        if kind not in _BLOCK:
            raise ValueError(f"{name}: unknown tensor type {kind}")
        block, size = _BLOCK[kind]
        n = int(np.prod(ne))
        if ne[0] % block or len(raw) != n // block * size:
            raise ValueError(f"{name}: {len(raw)} bytes do not match {kind} {tuple(ne)}")
        self._tensor(name, tuple(int(v) for v in ne), kind, bytes(raw))

    def add_lazy_tensor(self, name: str, ne, kind: str, produce):
        """A tensor whose bytes `produce()` returns when the file is written (one tensor in
        memory at a time, for multi-GB files)."""
        if kind not in _BLOCK:
            raise ValueError(f"{name}: unknown tensor type {kind}")
        block, _ = _BLOCK[kind]
        if ne[0] % block:
            raise ValueError(f"{name}: {tuple(ne)} is not whole {kind} blocks")
        self._tensor(name, tuple(int(v) for v in ne), kind, produce)

    def _tensor(self, name, ne, kind, raw):
        _check_name("tensor name", name)
        if name in self._names:
            raise ValueError(f"tensor {name!r} added twice")
        if not ne or len(ne) > 4 or any(v < 0 for v in ne):
            raise ValueError(f"{name}: dimensions {ne} are not 1 to 4 non-negative sizes")
        self._names.add(name)
        self.tensors.append((name, ne, kind, raw))

    def _nbytes(self, ne, kind):
        block, size = _BLOCK[kind]
        return int(np.prod(ne)) // block * size

    def write(self):
        head = b"GGUF" + struct.pack("<IQQ", 3, len(self.tensors), len(self.kv))
        for key, vtype, payload in self.kv:
            head += _str(key) + struct.pack("<I", vtype) + payload
        offsets, off = [], 0
        for _, ne, kind, _ in self.tensors:
            offsets.append(off)
            off += self._nbytes(ne, kind)
            off += -off % self.alignment
        for (name, ne, kind, _), o in zip(self.tensors, offsets):
            head += _str(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
            head += struct.pack("<IQ", GGML_TYPES[kind], o)
        head += b"\0" * (-len(head) % self.alignment)
        tmp = self.path.with_name(f"{self.path.name}.{os.getpid()}.tmp")
        try:
            with open(tmp, "wb") as f:
                f.write(head)
                for name, ne, kind, raw in self.tensors:
                    if callable(raw):
                        raw = raw()
                        if len(raw) != self._nbytes(ne, kind):
                            raise ValueError(f"{name}: produced {len(raw)} bytes, expected {self._nbytes(ne, kind)}")
                    f.write(raw)
                    f.write(b"\0" * (-len(raw) % self.alignment))
        except BaseException:
            tmp.unlink(missing_ok=True)  # a tensor that cannot be produced leaves no partial file
            raise
        os.replace(tmp, self.path)
        return self.path
