"""The GGUF reader (host code, no GPU) against files made by the package's writer."""
import ctypes
import struct

import numpy as np
import pytest

from sardyne_b200 import capi
from sardyne_b200.gguf_writer import GGUFWriter


def open_gguf(path):
    err = ctypes.create_string_buffer(256)
    h = capi.lib().gguf_open(str(path).encode(), err, len(err))
    return h, err.value.decode()


def test_roundtrip(tmp_path):
    w = GGUFWriter(tmp_path / "a.gguf")
    w.add("general.architecture", "llama")
    w.add("llama.block_count", 3)
    w.add("llama.rope.freq_base", 10000.0)
    w.add("tokenizer.ggml.tokens", ["a", "bé", ""])
    x = np.arange(64, dtype=np.float32).reshape(2, 32)
    w.add_tensor("t.weight", x)
    w.add_raw_tensor("q.weight", (32, 2), "Q8_0", bytes(range(68)))
    w.write()
    lib = capi.lib()
    h, err = open_gguf(w.path)
    assert h, err
    try:
        assert lib.gguf_version(h) == 3 and lib.gguf_n_kv(h) == 4 and lib.gguf_n_tensors(h) == 2
        i = lib.gguf_find_kv(h, b"llama.block_count")
        v = ctypes.c_uint64()
        assert lib.gguf_kv_get_u64(h, i, ctypes.byref(v)) == 0 and v.value == 3
        f = ctypes.c_double()
        assert lib.gguf_kv_get_f64(h, lib.gguf_find_kv(h, b"llama.rope.freq_base"), ctypes.byref(f)) == 0
        assert f.value == 10000.0
        n = ctypes.c_uint64()
        p = lib.gguf_kv_get_str(h, lib.gguf_find_kv(h, b"general.architecture"), ctypes.byref(n))
        assert ctypes.string_at(p, n.value) == b"llama"
        k = lib.gguf_find_kv(h, b"tokenizer.ggml.tokens")
        got = [ctypes.string_at(lib.gguf_kv_get_arr_str(h, k, j, ctypes.byref(n)), n.value).decode() for j in range(3)]
        assert got == ["a", "bé", ""]
        assert not lib.gguf_kv_get_arr_str(h, k, 3, ctypes.byref(n))
        assert lib.gguf_kv_get_u64(h, lib.gguf_find_kv(h, b"general.architecture"), ctypes.byref(v)) != 0
        t = lib.gguf_get_tensor(h, lib.gguf_find_tensor(h, b"t.weight")).contents
        assert (t.n_dims, tuple(t.ne[:2]), t.type, t.nbytes) == (2, (32, 2), 0, 256)
        assert np.array_equal(np.frombuffer(ctypes.string_at(t.data, t.nbytes), np.float32).reshape(2, 32), x)
        t = lib.gguf_get_tensor(h, lib.gguf_find_tensor(h, b"q.weight")).contents
        assert t.offset % 32 == 0 and ctypes.string_at(t.data, t.nbytes) == bytes(range(68))
        assert lib.gguf_type_name(14) == b"Q6_K" and lib.gguf_type_name(4) is None
        assert lib.gguf_find_tensor(h, b"nope") == -1
    finally:
        lib.gguf_close(h)


def _raw(path, kvs=(), tensors=(), version=3):
    def s(b):
        return struct.pack("<Q", len(b)) + b
    out = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kvs))
    for k, t, v in kvs:
        out += s(k) + struct.pack("<I", t) + v
    for n, ne, t, off in tensors:
        out += s(n) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne) + struct.pack("<IQ", t, off)
    out += b"\0" * (-len(out) % 32)
    path.write_bytes(out + b"\0" * 64 * max(1, len(tensors)))
    return path


@pytest.mark.parametrize("case,msg", [
    ("valid", None), ("nul_key", "UTF-8"), ("dup_key", "duplicato"), ("bad_utf8", "UTF-8"),
    ("overlong", "UTF-8"), ("surrogate", "UTF-8"), ("dup_tensor", "duplicato"), ("nul_name", "UTF-8"),
    ("zero_dim", "nulla"), ("big_endian", "big-endian"), ("bad_type", "sconosciuto"), ("bad_align", "alignment"),
    ("past_end", "oltre la fine"), ("unaligned", "allineato"), ("bad_block", "multiplo")])
def test_rejections(tmp_path, case, msg):
    U32 = 4
    kv = [(b"general.architecture", 8, struct.pack("<Q", 4) + b"test")]
    t = [(b"a", (4,), 0, 0)]
    if case == "nul_key":
        kv.append((b"k\0x", U32, struct.pack("<I", 1)))
    elif case == "dup_key":
        kv += [(b"k", U32, struct.pack("<I", 1)), (b"k", U32, struct.pack("<I", 2))]
    elif case == "bad_utf8":
        kv.append((b"caf\xe9", U32, struct.pack("<I", 1)))
    elif case == "overlong":
        kv.append((b"\xc0\xaf", U32, struct.pack("<I", 1)))
    elif case == "surrogate":
        kv.append((b"\xed\xa0\x80", U32, struct.pack("<I", 1)))
    elif case == "dup_tensor":
        t.append((b"a", (4,), 0, 32))
    elif case == "nul_name":
        t = [(b"a\0b", (4,), 0, 0)]
    elif case == "zero_dim":
        t = [(b"a", (4, 0), 0, 0)]
    elif case == "bad_type":
        t = [(b"a", (4,), 4, 0)]
    elif case == "bad_align":
        kv.append((b"general.alignment", U32, struct.pack("<I", 48)))
    elif case == "past_end":
        t = [(b"a", (4096,), 0, 0)]
    elif case == "unaligned":
        t = [(b"a", (4,), 0, 8)]
    elif case == "bad_block":
        t = [(b"a", (16,), 8, 0)]
    path = _raw(tmp_path / f"{case}.gguf", kv, t, version=0x03000000 if case == "big_endian" else 3)
    h, err = open_gguf(path)
    if msg is None:
        assert h, err
        capi.lib().gguf_close(h)
    else:
        assert not h and msg in err


def test_missing_and_truncated(tmp_path):
    h, err = open_gguf(tmp_path / "missing.gguf")
    assert not h and "impossibile aprire" in err
    w = GGUFWriter(tmp_path / "a.gguf")
    w.add("general.architecture", "llama")
    w.add_tensor("t.weight", np.ones((4, 32), np.float32))
    w.write()
    data = w.path.read_bytes()
    for cut in (3, 20, 60, len(data) - 8):
        p = tmp_path / f"cut{cut}.gguf"
        p.write_bytes(data[:cut])
        h, err = open_gguf(p)
        assert not h and err


def test_writer_refuses_what_readers_reject(tmp_path):
    """The package's GGUF writer refuses input that would make an unreadable or ambiguous file
    (the rules of the reference's writer, tests/test_gguf.py:412-437), and widens integer arrays."""
    with pytest.raises(ValueError):
        GGUFWriter(tmp_path / "x.gguf", alignment=24)  # not a power of two
    w = GGUFWriter(tmp_path / "x.gguf")
    w.add("k", 1)
    bad = [lambda: w.add("k", 2),                       # key added twice
           lambda: w.add("a\0b", 1),                    # NUL in a key
           lambda: w.add("", 1),                        # empty key
           lambda: w.add("big", 2 ** 64),               # beyond 64 bits
           lambda: w.add("u8", 256, 0),                 # beyond UINT8
           lambda: w.add("mix", [1, "a"]),              # mixed array
           lambda: w.add("nested", [[1, 2], [3]]),      # array of arrays
           lambda: w.add("obj", object()),
           lambda: w.add_raw_tensor("q", (32,), "Q8_0", b"\0" * 33),  # Q8_0 holds 34 bytes per 32
           lambda: w.add_raw_tensor("z", (32,), "Q9_9", b""),         # unknown type
           lambda: w.add_tensor("n\0", np.ones(4, np.float32))]
    for fn in bad:
        with pytest.raises((ValueError, TypeError)):
            fn()
    w.add("np_scalar", np.float32(1.5))
    w.add("wide", [1, 2 ** 33])
    w.add("neg", [-1, 2 ** 40])
    w.add_tensor("t", np.ones(4, np.float32))
    with pytest.raises(ValueError):
        w.add_tensor("t", np.ones(4, np.float32))       # tensor name added twice
    lib = capi.lib()
    err = ctypes.create_string_buffer(256)
    h = lib.gguf_open(str(w.write()).encode(), err, len(err))
    assert h, err.value
    try:
        kv = {lib.gguf_get_kv(h, i).contents.key.decode(): lib.gguf_get_kv(h, i).contents for i in range(lib.gguf_n_kv(h))}
        assert (kv["wide"].type, kv["wide"].arr_type, kv["wide"].n) == (9, 10, 2)  # UINT64 array
        assert (kv["neg"].type, kv["neg"].arr_type) == (9, 11)                    # INT64 array
        assert kv["np_scalar"].type == 6 and lib.gguf_n_tensors(h) == 1
    finally:
        lib.gguf_close(h)
    w2 = GGUFWriter(tmp_path / "a64.gguf", alignment=64)  # a non-default alignment is recorded
    w2.add_tensor("t", np.ones(3, np.float32))
    h = lib.gguf_open(str(w2.write()).encode(), err, len(err))
    assert h, err.value
    assert lib.gguf_alignment(h) == 64
    lib.gguf_close(h)


def test_writer_failure_leaves_the_existing_file(tmp_path):
    """A tensor that cannot be produced while the file is written leaves the previous file intact
    and no temporary file (reference tests/test_gguf.py:440-461)."""
    path = tmp_path / "m.gguf"
    w = GGUFWriter(path)
    w.add_tensor("t", np.arange(8, dtype=np.float32))
    before = w.write().read_bytes()

    def boom():
        raise RuntimeError("cannot produce")

    w2 = GGUFWriter(path)
    w2.add_lazy_tensor("t", (4,), "F32", boom)
    with pytest.raises(RuntimeError):
        w2.write()
    assert path.read_bytes() == before and [p.name for p in tmp_path.iterdir()] == ["m.gguf"]
