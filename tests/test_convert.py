"""The HF -> GGUF converter with K-quants (sardyne_b200.convert), on the CPU.

Tiny llama / qwen2 / qwen3moe checkpoints are written as safetensors here. Checked:
  * at every type the reference's own converter writes (sardyne/loader/convert.py: f32, f16, bf16,
    q8_0, q4_0) the output equals its output tensor for tensor, byte for byte (names, types,
    shapes, llama's q/k row order), with every metadata entry equal (the reference's converter has
    no MoE, so qwen3moe is checked against its checkpoint directly);
  * in the Q4_K_M mix every tensor gets the type the mix names, and dequantizes (oracle) to the
    checkpoint's weights within the reference's own error bounds for published files
    (tests/test_quant.py:53: Q4_K < 0.11, Q6_K < 0.03, Q5_0 < 0.07 relative RMS; Q8_0 < 0.01);
  * the reference engine (oracle/_ref) runs the Q4_K_M file, and its logits follow those of the F32
    file (the quantization error only).
"""
import ctypes
import json
import struct

import numpy as np
import pytest

import oracle
import refruntime as rt
from sardyne_b200 import capi, convert, synth

BOUND = {"Q4_K": 0.11, "Q6_K": 0.03, "Q5_0": 0.07, "Q8_0": 0.01, "F32": 0.0, "F16": 1e-3}


def write_safetensors(path, tensors, dtype="F32"):
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a, np.float32)
        raw = ((a.view(np.uint32) + 0x8000) >> 16).astype(np.uint16).tobytes() if dtype == "BF16" else \
            a.astype(np.float16).tobytes() if dtype == "F16" else a.tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    path.write_bytes(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def checkpoint(tmp_path, arch, tied, dtype="F32"):
    rng = np.random.default_rng(len(arch))
    dim, n_head, n_kv, hd, ffn, vocab, n_layer = 256, 4, 2, 64, 512, 96, 2
    hf = {"llama": "LlamaForCausalLM", "qwen2": "Qwen2ForCausalLM", "qwen3": "Qwen3ForCausalLM",
          "qwen3moe": "Qwen3MoeForCausalLM"}[arch]
    cfg = {"architectures": [hf], "hidden_size": dim, "num_hidden_layers": n_layer, "num_attention_heads": n_head,
           "num_key_value_heads": n_kv, "intermediate_size": ffn, "vocab_size": vocab, "rms_norm_eps": 1e-6,
           "rope_theta": 10000.0, "max_position_embeddings": 128, "tie_word_embeddings": tied,
           "bos_token_id": 1, "eos_token_id": 2 if arch != "qwen3" else [2, 4]}
    if arch == "qwen3moe":
        cfg.update(num_experts=4, num_experts_per_tok=2, moe_intermediate_size=256, head_dim=hd)
    if arch == "qwen3":
        cfg.update(head_dim=hd)
    t = {"model.embed_tokens.weight": rng.standard_normal((vocab, dim)) * 0.02,
         "model.norm.weight": 1 + rng.standard_normal(dim) * 0.1}
    if not tied:
        t["lm_head.weight"] = rng.standard_normal((vocab, dim)) * 0.02
    for i in range(n_layer):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = 1 + rng.standard_normal(dim) * 0.1
        t[p + "post_attention_layernorm.weight"] = 1 + rng.standard_normal(dim) * 0.1
        t[p + "self_attn.q_proj.weight"] = rng.standard_normal((n_head * hd, dim)) * 0.02
        t[p + "self_attn.k_proj.weight"] = rng.standard_normal((n_kv * hd, dim)) * 0.02
        t[p + "self_attn.v_proj.weight"] = rng.standard_normal((n_kv * hd, dim)) * 0.02
        t[p + "self_attn.o_proj.weight"] = rng.standard_normal((dim, n_head * hd)) * 0.02
        if arch == "qwen2":
            for n, r in (("q", n_head * hd), ("k", n_kv * hd), ("v", n_kv * hd)):
                t[p + f"self_attn.{n}_proj.bias"] = rng.standard_normal(r) * 0.1
        if arch in ("qwen3", "qwen3moe"):
            t[p + "self_attn.q_norm.weight"] = 1 + rng.standard_normal(hd) * 0.1
            t[p + "self_attn.k_norm.weight"] = 1 + rng.standard_normal(hd) * 0.1
        if arch == "qwen3moe":
            t[p + "mlp.gate.weight"] = rng.standard_normal((4, dim)) * 0.1
            for e in range(4):
                t[p + f"mlp.experts.{e}.gate_proj.weight"] = rng.standard_normal((256, dim)) * 0.02
                t[p + f"mlp.experts.{e}.up_proj.weight"] = rng.standard_normal((256, dim)) * 0.02
                t[p + f"mlp.experts.{e}.down_proj.weight"] = rng.standard_normal((dim, 256)) * 0.02
        else:
            t[p + "mlp.gate_proj.weight"] = rng.standard_normal((ffn, dim)) * 0.02
            t[p + "mlp.up_proj.weight"] = rng.standard_normal((ffn, dim)) * 0.02
            t[p + "mlp.down_proj.weight"] = rng.standard_normal((dim, ffn)) * 0.02
    d = tmp_path / f"{arch}-{'tied' if tied else 'untied'}-{dtype}"
    d.mkdir()
    (d / "config.json").write_text(json.dumps(cfg))
    if arch == "qwen2":  # end ids from generation_config.json take precedence
        (d / "generation_config.json").write_text(json.dumps({"eos_token_id": [5, 2]}))
    write_safetensors(d / "model.safetensors", t, dtype)
    return d


def read_gguf(path):
    """{name: (type name, ne, bytes)} and {key: value} through this library's reader (strings and
    string arrays as str; other arrays as (element type, raw bytes); scalars as (GGUF type, value))."""
    lib = capi.lib()
    err = ctypes.create_string_buffer(256)
    h = lib.gguf_open(str(path).encode(), err, len(err))
    assert h, err.value
    tensors, kvs = {}, {}
    try:
        for i in range(lib.gguf_n_tensors(h)):
            t = lib.gguf_get_tensor(h, i).contents
            tensors[t.name.decode()] = (lib.gguf_type_name(t.type).decode(), tuple(t.ne[:t.n_dims]),
                                        ctypes.string_at(t.data, t.nbytes))
        for i in range(lib.gguf_n_kv(h)):
            kv = lib.gguf_get_kv(h, i).contents
            key = kv.key.decode()
            if kv.type == 8:
                n = ctypes.c_uint64()
                kvs[key] = ctypes.string_at(lib.gguf_kv_get_str(h, i, ctypes.byref(n)), n.value).decode()
            elif kv.type == 9 and kv.arr_type == 8:  # array of strings
                n = ctypes.c_uint64()
                kvs[key] = [ctypes.string_at(lib.gguf_kv_get_arr_str(h, i, j, ctypes.byref(n)), n.value).decode()
                            for j in range(kv.n)]
            elif kv.type == 9:  # array of 4-byte integers
                kvs[key] = (kv.arr_type, ctypes.string_at(kv.ptr, 4 * kv.n))
            else:
                v = ctypes.c_double()
                u = ctypes.c_uint64()
                kvs[key] = (kv.type, u.value if lib.gguf_kv_get_u64(h, i, ctypes.byref(u)) == 0 else
                            (v.value if lib.gguf_kv_get_f64(h, i, ctypes.byref(v)) == 0 else None))
    finally:
        lib.gguf_close(h)
    return tensors, kvs


def floats(kind, ne, raw):
    n_in = ne[0]
    if kind == "F32":
        return np.frombuffer(raw, np.float32).reshape(-1, n_in)
    if kind == "F16":
        return np.frombuffer(raw, np.float16).astype(np.float32).reshape(-1, n_in)
    return oracle.dequant(np.frombuffer(raw, np.uint8), kind, n_in)


@pytest.mark.skipif(not rt.available(), reason="the reference's Python package is not installed")
@pytest.mark.parametrize("outtype", ["f32", "f16", "bf16", "q8_0", "q4_0"])
@pytest.mark.parametrize("arch,tied,dtype", [("llama", True, "F32"), ("qwen2", False, "F32"), ("qwen3", True, "F32"),
                                             ("qwen2", False, "BF16"), ("llama", True, "F16")])
def test_equals_the_reference_converter(tmp_path, arch, tied, dtype, outtype):
    """At every type the reference's converter writes (sardyne/loader/convert.py:30-31), from
    checkpoints stored in F32, BF16 or F16, every tensor (name, type, shape, bytes) and every
    metadata entry equal its output."""
    rt.modules()
    from sardyne.loader import convert as ref_convert  # the reference's converter
    ck = checkpoint(tmp_path, arch, tied, dtype)
    ours = convert.convert(ck, tmp_path / "ours.gguf", outtype)
    ref_convert.convert(ck, tmp_path / "ref.gguf", outtype)
    a, akv = read_gguf(ours)
    b, bkv = read_gguf(tmp_path / "ref.gguf")
    assert a.keys() == b.keys()
    for name in a:
        assert a[name] == b[name], name
    assert akv == bkv


@pytest.mark.parametrize("arch,tied,dtype", [("llama", True, "F32"), ("qwen2", False, "BF16"),
                                             ("qwen3moe", False, "F32")])
def test_q4_k_m_mix_and_error_bounds(tmp_path, arch, tied, dtype):
    ck = checkpoint(tmp_path, arch, tied, dtype)
    f32, _ = read_gguf(convert.convert(ck, tmp_path / "f32.gguf", "f32"))
    q, kv = read_gguf(convert.convert(ck, tmp_path / "q.gguf", "q4_k_m"))
    assert kv["general.file_type"][1] == 15 and q.keys() == f32.keys()
    mix = synth.mix_q4_k_m_tied if tied else synth.mix_q4_k_m_untied
    for name, (kind, ne, raw) in q.items():
        want_kind = "F32" if len(ne) == 1 or "gate_inp" in name else mix(name, ne[0])
        assert kind == want_kind, name
        ref = floats(*f32[name])
        got = floats(kind, ne, raw)
        rel = np.sqrt(np.mean((got - ref) ** 2) / np.mean(ref ** 2))
        assert rel <= BOUND[kind], (name, kind, rel)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")
@pytest.mark.parametrize("arch,tied,min_corr", [("llama", True, 0.99), ("qwen3moe", False, 0.97)])
def test_reference_engine_runs_the_conversion(tmp_path, arch, tied, min_corr):
    """(The MoE model's bound is lower: its router picks 2 of 4 experts, and the quantization noise
    can change a pick.)"""
    ck = checkpoint(tmp_path, arch, tied)
    tokens = [3, 14, 15, 9, 26, 5, 35, 8]
    out = {}
    for outtype in ("f32", "q4_k_m"):
        path = convert.convert(ck, tmp_path / f"{outtype}.gguf", outtype)
        m = rt.model(path, oracle.REF_LIB)
        out[outtype] = rt.Context(m, max_seq=32, n_batch=8, logits_all=True).eval(tokens)
    a, b = out["f32"].ravel(), out["q4_k_m"].ravel()
    assert np.isfinite(b).all()
    assert np.corrcoef(a, b)[0, 1] > min_corr


def write_tokenizer(directory, style, split_regex=None):
    """A small byte-level BPE tokenizer.json (+ tokenizer_config.json) of the two pre-tokenizer
    styles the reference's converter accepts."""
    vocab = {t: i for i, t in enumerate(["a", "b", "c", "ab", "abc", "\u0120", "\u0120a", "1", "2", "x"])}
    merges = [["a", "b"], ["ab", "c"], ["\u0120", "a"]]
    if style == "qwen2":
        pre = {"type": "Sequence", "pretokenizers": [
            {"type": "Split", "pattern": {"Regex": split_regex}, "behavior": "Isolated", "invert": False},
            {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": False, "use_regex": False}]}
        norm = {"type": "NFC"}
        merges = [" ".join(m) for m in merges]
    else:
        pre = {"type": "Sequence", "pretokenizers": [
            {"type": "Digits", "individual_digits": True},
            {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True, "use_regex": True}]}
        norm = None
    tok = {"version": "1.0", "added_tokens": [
        {"id": 10, "content": "<|endoftext|>", "special": True},
        {"id": 12, "content": "<tool>", "special": False}],
        "normalizer": norm, "pre_tokenizer": pre,
        "model": {"type": "BPE", "vocab": vocab, "merges": merges}}
    (directory / "tokenizer.json").write_text(json.dumps(tok))
    if style == "qwen2":
        (directory / "tokenizer_config.json").write_text(json.dumps(
            {"chat_template": "{% for m in messages %}{{ m['content'] }}{% endfor %}"}))


@pytest.mark.skipif(not rt.available(), reason="the reference's Python package is not installed")
@pytest.mark.parametrize("arch,tied,style", [("qwen2", False, "qwen2"), ("llama", True, "smollm")])
def test_tokenizer_metadata_equals_the_reference_converter(tmp_path, arch, tied, style):
    """With a tokenizer.json beside the checkpoint, every tokenizer.* key (tokens with [PADn] up to
    the model's vocabulary, token types, merges, pre-tokenizer name, chat template) equals the
    reference's converter's (sardyne/loader/convert.py:105-116)."""
    rt.modules()
    from sardyne.loader import convert as ref_convert  # the reference's converter
    from sardyne.tokenizer import bpe as ref_bpe       # its pre-tokenizer regex
    assert convert.QWEN2_SPLIT == ref_bpe._QWEN2
    ck = checkpoint(tmp_path, arch, tied)
    write_tokenizer(ck, style, convert.QWEN2_SPLIT)
    _, akv = read_gguf(convert.convert(ck, tmp_path / "ours.gguf", "q4_k_m"))
    ref_convert.convert(ck, tmp_path / "ref.gguf", "f32")
    _, bkv = read_gguf(tmp_path / "ref.gguf")
    want = {k: v for k, v in bkv.items() if k.startswith("tokenizer.")}
    assert {"tokenizer.ggml.tokens", "tokenizer.ggml.token_type", "tokenizer.ggml.merges",
            "tokenizer.ggml.pre"} <= set(want)
    assert len(want["tokenizer.ggml.tokens"]) == 96 and want["tokenizer.ggml.tokens"][95] == "[PAD95]"
    for key, value in want.items():
        assert akv.get(key) == value, key
    assert set(k for k in akv if k.startswith("tokenizer.")) == set(want)
    # the reference's text front-end reads the file: its tokenizer loaded from our GGUF encodes like
    # the same tokenizer loaded from tokenizer.json (special tokens, digits, spaces, unknown bytes)
    from sardyne.tokenizer.bpe import BPETokenizer
    ours = BPETokenizer.load(model=tmp_path / "ours.gguf")
    hf = BPETokenizer.load(hf_dir=ck)
    # a GGUF keeps one end id (the first), so the end ids are those of the reference's own file
    assert ours.pre == hf.pre == style and ours.eos_ids == BPETokenizer.load(model=tmp_path / "ref.gguf").eos_ids
    for text in ["abc ab a", "a12 cab<|endoftext|>abc<tool> x", " a  abc\nb", "zz\u00e9 12"]:
        assert ours.encode(text) == hf.encode(text), text
        assert ours.decode(ours.encode(text)) == hf.decode(hf.encode(text))


@pytest.mark.skipif(not rt.available(), reason="the reference's Python package is not installed")
def test_unsupported_pretokenizers_are_refused_like_the_reference(tmp_path):
    """A split regex other than Qwen2's, or a tokenizer model other than BPE, is refused by both
    converters (sardyne/tokenizer/bpe.py:104-105,192-201) instead of being written under a
    pre-tokenizer name that would tokenize differently."""
    rt.modules()
    from sardyne.loader import convert as ref_convert
    ck = checkpoint(tmp_path, "qwen2", False)
    write_tokenizer(ck, "qwen2", r"\p{L}+|\s+")
    with pytest.raises(NotImplementedError):
        convert.convert(ck, tmp_path / "ours.gguf", "f32")
    assert not list(tmp_path.glob("ours.gguf*"))  # nothing written, not even a temporary file
    with pytest.raises(NotImplementedError):
        ref_convert.convert(ck, tmp_path / "ref.gguf", "f32")
    tok = json.loads((ck / "tokenizer.json").read_text())
    tok["model"]["type"] = "Unigram"
    (ck / "tokenizer.json").write_text(json.dumps(tok))
    with pytest.raises(NotImplementedError):
        convert.convert(ck, tmp_path / "ours.gguf", "f32")
    with pytest.raises(NotImplementedError):
        ref_convert.convert(ck, tmp_path / "ref.gguf", "f32")


@pytest.mark.skipif(not rt.available(), reason="the reference's Python package is not installed")
def test_f16_overflow_is_refused_like_the_reference(tmp_path):
    """A matrix value beyond the f16 range is refused at f16 (the reference's message names the
    tensor and "f16"), leaving neither the output nor a temporary file; bf16 converts it
    (reference tests/test_convert.py:142-152)."""
    rt.modules()
    from sardyne.loader import convert as ref_convert
    ck = checkpoint(tmp_path, "llama", True)
    raw = (ck / "model.safetensors").read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    off = json.loads(raw[8:8 + n])["model.layers.0.mlp.up_proj.weight"]["data_offsets"][0] + 8 + n
    (ck / "model.safetensors").write_bytes(raw[:off] + struct.pack("<f", 70000.0) + raw[off + 4:])
    out = tmp_path / "out"
    out.mkdir()
    for fn, name in ((convert.convert, "ours.gguf"), (ref_convert.convert, "ref.gguf")):
        with pytest.raises(ValueError, match="blk.0.ffn_up.weight.*f16"):
            fn(ck, out / name, "f16")
    assert not list(out.iterdir())
    a, _ = read_gguf(convert.convert(ck, out / "ours.gguf", "bf16"))
    ref_convert.convert(ck, out / "ref.gguf", "bf16")
    assert a == read_gguf(out / "ref.gguf")[0]


ROPE_CASES = [{}, {"rope_theta": 5e5}, {"rope_parameters": {"rope_theta": 1e4, "rope_type": "yarn"}},
              {"rope_parameters": {"full_attention": {"rope_theta": 3.0}}},
              {"rope_scaling": {"rope_type": "llama3", "factor": 8.0}}, {"rope_scaling": {"type": "linear", "factor": 2.0}},
              {"rope_scaling": None, "rope_theta": 1e6}, {"rope_parameters": {"rope_theta": 2e4, "rope_type": "default"}},
              {"rope_scaling": {"rope_type": "default"}, "rope_theta": 7.0},
              {"rope_parameters": {"sliding_attention": {"rope_theta": 1.0}}},
              {"rope_parameters": {"full_attention": {"rope_theta": 2.0}, "sliding_attention": {"rope_theta": 1.0}}},
              {"rope_parameters": {"rope_type": None, "rope_theta": 9.0}}]


@pytest.mark.skipif(not rt.available(), reason="the reference's Python package is not installed")
@pytest.mark.parametrize("cfg", ROPE_CASES)
def test_rope_theta_and_scaling_refusals_match_the_reference(cfg):
    """The RoPE base read from config.json, and the refusal of scaled RoPE variants, as the
    reference's hf_config.rope_theta (reference tests/test_convert.py:112-121)."""
    rt.modules()
    from sardyne.loader import hf_config

    def outcome(fn):
        try:
            return fn(cfg)
        except NotImplementedError:
            return "refused"
    assert outcome(convert.rope_theta) == outcome(hf_config.rope_theta)


def _st_file(directory, header, data=b"", header_len=None):
    directory.mkdir()
    h = json.dumps(header).encode()
    (directory / "m.safetensors").write_bytes(struct.pack("<Q", len(h) if header_len is None else header_len) + h + data)
    return directory


@pytest.mark.parametrize("header,data", [
    ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [-8, 0]}}, b"\0" * 8),   # negative offset
    ({"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, b"\0" * 8),   # past the file
    ({"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8),    # shape and size differ
    ({"a": {"dtype": "F8_E4M3", "shape": [8], "data_offsets": [0, 8]}}, b"\0" * 8),  # unknown dtype
    ({"a": {"dtype": "F32", "shape": [-2], "data_offsets": [0, 8]}}, b"\0" * 8),   # negative dimension
    ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0]}}, b"\0" * 8),       # one offset
    ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [8, 0]}}, b"\0" * 8),    # end before begin
    ({"a": "x"}, b""),                                                             # entry not an object
    ([1, 2], b""),                                                                 # header not an object
])
def test_safetensors_headers_are_checked_when_opened(tmp_path, header, data):
    """The converter's safetensors reader refuses a header that does not describe its data (the
    cases of reference tests/test_safetensors.py:29-41) with SafeTensorsError, a ValueError."""
    with pytest.raises(convert.SafeTensorsError):
        convert.SafeTensors(_st_file(tmp_path / "ck", header, data))


def test_safetensors_lengths_and_json(tmp_path):
    (tmp_path / "short").mkdir()
    (tmp_path / "short" / "m.safetensors").write_bytes(b"\1\2\3")
    with pytest.raises(convert.SafeTensorsError):
        convert.SafeTensors(tmp_path / "short")
    with pytest.raises(convert.SafeTensorsError):  # a huge header length allocates nothing
        convert.SafeTensors(_st_file(tmp_path / "huge", {}, header_len=2 ** 62))
    (tmp_path / "json").mkdir()
    (tmp_path / "json" / "m.safetensors").write_bytes(struct.pack("<Q", 3) + b"{x}")
    with pytest.raises(convert.SafeTensorsError):
        convert.SafeTensors(tmp_path / "json")
    ok = convert.SafeTensors(_st_file(tmp_path / "ok", {"a": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, 24]}},
                                      np.arange(6, dtype=np.float32).tobytes()))
    assert ok.shape("a") == (2, 3) and np.array_equal(ok.get("a"), np.arange(6, dtype=np.float32).reshape(2, 3))


def shard_checkpoint(ck, out):
    """The checkpoint `ck` split over two shards with a model.safetensors.index.json, in `out`."""
    out.mkdir()
    for meta in ck.glob("*.json"):
        (out / meta.name).write_text(meta.read_text())
    st = convert.SafeTensors(ck)
    names = sorted(st.index)
    halves = {"model-00001-of-00002.safetensors": names[::2], "model-00002-of-00002.safetensors": names[1::2]}
    for fname, part in halves.items():
        write_safetensors(out / fname, {n: st.get(n) for n in part})
    (out / "model.safetensors.index.json").write_text(json.dumps(
        {"metadata": {}, "weight_map": {n: f for f, part in halves.items() for n in part}}))
    return out


@pytest.mark.skipif(not rt.available(), reason="the reference's Python package is not installed")
def test_sharded_checkpoint_converts_like_the_single_file(tmp_path):
    rt.modules()
    from sardyne.loader import convert as ref_convert
    ck = checkpoint(tmp_path, "qwen2", False)
    sh = shard_checkpoint(ck, tmp_path / "sharded")
    a, akv = read_gguf(convert.convert(ck, tmp_path / "single.gguf", "q8_0"))
    b, bkv = read_gguf(convert.convert(sh, tmp_path / "sharded.gguf", "q8_0"))
    ref_convert.convert(sh, tmp_path / "ref.gguf", "q8_0")
    c, ckv = read_gguf(tmp_path / "ref.gguf")
    assert a == b and b == c and bkv == ckv
    assert {k: v for k, v in akv.items() if k != "general.name"} == {k: v for k, v in bkv.items() if k != "general.name"}


def test_shard_index_is_checked(tmp_path):
    """Index entries must name files of the model directory that hold the tensor (reference
    tests/test_safetensors.py:51-62); without an index a tensor name may appear in one file only."""
    ck = checkpoint(tmp_path, "llama", True)
    sh = shard_checkpoint(ck, tmp_path / "sharded")
    index = json.loads((sh / "model.safetensors.index.json").read_text())
    name = next(iter(index["weight_map"]))
    for bad in ("../outside.safetensors", "/abs/model.safetensors", "model.bin"):
        (sh / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {**index["weight_map"], name: bad}}))
        with pytest.raises(convert.SafeTensorsError, match="not a file of the model directory"):
            convert.SafeTensors(sh)
    other = next(f for f in set(index["weight_map"].values()) if f != index["weight_map"][name])
    (sh / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {**index["weight_map"], name: other}}))
    with pytest.raises(convert.SafeTensorsError, match="does not hold it"):
        convert.SafeTensors(sh)
    (sh / "model.safetensors.index.json").unlink()
    write_safetensors(sh / "extra.safetensors", {name: np.zeros(convert.SafeTensors(ck).shape(name), np.float32)})
    with pytest.raises(convert.SafeTensorsError, match="also in another file"):
        convert.SafeTensors(sh)
