"""Hugging Face checkpoint (config.json + *.safetensors) to GGUF, in the block formats this library
runs, K-quants included.

    python -m sardyne_b200.convert HF_DIR OUT.gguf [--outtype q4_k_m|q6_k|q4_k|q8_0|q4_0|bf16|f16|f32]

The reference's converter (sardyne/loader/convert.py:31,78-103) writes F32/F16/BF16/Q8_0/Q4_0 of the
dense architectures only; this one adds the K-quants, in particular the Q4_K_M mix the BASELINE
models use (sardyne_b200.synth.q4_k_m: Q4_K by default, Q6_K on attn_v, on the ffn_down of even
layers and on the output matrix; rows that are not whole 256-element superblocks fall back to Q5_0
and Q8_0), and Qwen3-MoE checkpoints (the experts' matrices stacked into the GGUF expert tensors).
It follows the GGUF conventions the engine reads (tensor names, metadata keys, llama's q/k rows
reordered for RoPE on adjacent pairs); norms, biases and the MoE router stay F32. When the
directory holds a byte-level BPE tokenizer.json, the tokenizer goes into the file under the keys
the reference's text front-ends read (tokens, token types, merges, pre-tokenizer name, chat
template; reference sardyne/loader/convert.py:105-116), so its CLI and server run on the result.
Tensors are read, converted and written one at a time.
"""
import argparse
import json
import mmap
import pathlib
import struct

import numpy as np

from . import kquant, synth
from .gguf_writer import ARRAY, I32, STRING, GGUFWriter, f32_to_bf16

ARCHS = {"LlamaForCausalLM": "llama", "Qwen2ForCausalLM": "qwen2", "Qwen3ForCausalLM": "qwen3",
         "Qwen3MoeForCausalLM": "qwen3moe"}
# general.file_type values (the llama_ftype numbering GGUF readers use)
FILE_TYPES = {"f32": 0, "f16": 1, "q4_0": 2, "q8_0": 7, "q4_k": 14, "q4_k_m": 15, "q6_k": 18, "bf16": 32}

# tensors below model.layers.<i>.: HF suffix -> GGUF suffix below blk.<i>.
LAYER_TENSORS = (
    ("input_layernorm.weight", "attn_norm.weight"),
    ("post_attention_layernorm.weight", "ffn_norm.weight"),
    ("self_attn.q_proj.weight", "attn_q.weight"),
    ("self_attn.k_proj.weight", "attn_k.weight"),
    ("self_attn.v_proj.weight", "attn_v.weight"),
    ("self_attn.o_proj.weight", "attn_output.weight"),
    ("self_attn.q_proj.bias", "attn_q.bias"),
    ("self_attn.k_proj.bias", "attn_k.bias"),
    ("self_attn.v_proj.bias", "attn_v.bias"),
    ("self_attn.q_norm.weight", "attn_q_norm.weight"),
    ("self_attn.k_norm.weight", "attn_k_norm.weight"),
    ("mlp.gate_proj.weight", "ffn_gate.weight"),
    ("mlp.up_proj.weight", "ffn_up.weight"),
    ("mlp.down_proj.weight", "ffn_down.weight"),
    ("mlp.gate.weight", "ffn_gate_inp.weight"),
)
# MoE experts: mlp.experts.<e>.<HF> of every expert stacked into one GGUF tensor
EXPERT_TENSORS = (("gate_proj.weight", "ffn_gate_exps.weight"), ("up_proj.weight", "ffn_up_exps.weight"),
                  ("down_proj.weight", "ffn_down_exps.weight"))
MODEL_TENSORS = (("model.embed_tokens.weight", "token_embd.weight"), ("model.norm.weight", "output_norm.weight"),
                 ("lm_head.weight", "output.weight"))

_ST_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "F64": np.float64}

# GGUF token types (the llama.cpp numbering the reference's tokenizer reads)
TOKEN_NORMAL, TOKEN_CONTROL, TOKEN_USER_DEFINED, TOKEN_UNUSED = 1, 3, 4, 5

# The split pattern of Qwen2's byte-level BPE tokenizer.json (a published format constant); the
# reference's tokenizer reproduces exactly this pattern under the name "qwen2"
# (sardyne/tokenizer/bpe.py:28-29).
QWEN2_SPLIT = ("(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n]*"
               "|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+")


# The pre-tokenizers the reference's tokenizer reproduces (sardyne/tokenizer/bpe.py:192-201), as
# (pre-tokenizer step types, normalizer type, check of the first step, tokenizer.ggml.pre).
PRETOKENIZERS = (
    (("Split", "ByteLevel"), "NFC", lambda step: (step.get("pattern") or {}).get("Regex") == QWEN2_SPLIT, "qwen2"),
    (("Digits", "ByteLevel"), None, lambda step: bool(step.get("individual_digits")), "smollm"),
)


def pretokenizer_name(t: dict) -> str:
    """tokenizer.ggml.pre of a tokenizer.json whose pre-tokenizer is one of PRETOKENIZERS; any
    other is refused (NotImplementedError)."""
    sequence = (t.get("pre_tokenizer") or {}).get("pretokenizers") or []
    types = tuple(step.get("type") for step in sequence)
    normalizer = (t.get("normalizer") or {}).get("type")
    for want_types, want_normalizer, first_ok, name in PRETOKENIZERS:
        if types == want_types and normalizer == want_normalizer and first_ok(sequence[0]):
            return name
    raise NotImplementedError(f"pre-tokenizer {list(types)} with normalizer {normalizer} is not supported")


def tokenizer_fields(hf_dir: pathlib.Path, vocab_size: int) -> dict:
    """The GGUF tokenizer keys of a byte-level BPE tokenizer.json: one token per id up to the
    model's vocabulary size (vocabulary entries NORMAL, added tokens CONTROL when special else
    USER_DEFINED, ids no entry names "[PAD<id>]" and UNUSED), merges as "left right" strings, and
    the chat template of tokenizer_config.json when there is one."""
    t = json.loads((hf_dir / "tokenizer.json").read_text(encoding="utf-8"))
    model = t.get("model") or {}
    if model.get("type") != "BPE":
        raise NotImplementedError(f"tokenizer model {model.get('type')} is not supported")
    # id -> (text, type); added tokens override vocabulary entries of the same id
    table = {i: (tok, TOKEN_NORMAL) for tok, i in model["vocab"].items()}
    for a in t.get("added_tokens", []):
        table[a["id"]] = (a["content"], TOKEN_CONTROL if a.get("special") else TOKEN_USER_DEFINED)
    rows = [table.get(i, (f"[PAD{i}]", TOKEN_UNUSED)) for i in range(max(vocab_size, max(table) + 1))]
    # merges come as "left right" strings (older files) or as [left, right] pairs (newer ones)
    merges = [m if isinstance(m, str) else f"{m[0]} {m[1]}" for m in model.get("merges", [])]
    fields = {"tokenizer.ggml.model": "gpt2", "tokenizer.ggml.pre": pretokenizer_name(t),
              "tokenizer.ggml.tokens": [text for text, _ in rows],
              "tokenizer.ggml.token_type": [kind for _, kind in rows],
              "tokenizer.ggml.merges": merges}
    cfg_path = hf_dir / "tokenizer_config.json"
    cfg = json.loads(cfg_path.read_text(encoding="utf-8")) if cfg_path.exists() else {}
    if cfg.get("chat_template"):
        fields["tokenizer.chat_template"] = cfg["chat_template"]
    return fields


class SafeTensorsError(ValueError):
    """A .safetensors file whose header does not describe its data."""


def _check_entry(where: str, info, data_len: int) -> tuple:
    """(dtype, shape, begin, end) of one header entry, or SafeTensorsError: a known dtype,
    non-negative integer dimensions, two offsets inside the data, and as many bytes as the shape
    needs."""
    if not isinstance(info, dict):
        raise SafeTensorsError(f"{where}: entry is not an object")
    dtype, shape, offs = info.get("dtype"), info.get("shape"), info.get("data_offsets")
    if dtype not in _ST_DTYPES:
        raise SafeTensorsError(f"{where}: dtype {dtype} not supported")
    if not isinstance(shape, list) or not all(type(d) is int and d >= 0 for d in shape):
        raise SafeTensorsError(f"{where}: bad shape {shape!r}")
    if not isinstance(offs, list) or len(offs) != 2 or not all(type(o) is int for o in offs):
        raise SafeTensorsError(f"{where}: bad data_offsets {offs!r}")
    b, e = offs
    if not 0 <= b <= e <= data_len:
        raise SafeTensorsError(f"{where}: data [{b}, {e}) outside the file's {data_len} data bytes")
    if e - b != int(np.prod(shape, dtype=np.int64)) * np.dtype(_ST_DTYPES[dtype]).itemsize:
        raise SafeTensorsError(f"{where}: {e - b} bytes do not hold shape {shape} of {dtype}")
    return dtype, tuple(shape), b, e


class SafeTensors:
    """The tensors of a Hugging Face checkpoint directory, mapped read-only; get() returns float32.
    With model.safetensors.index.json the shards it names (plain file names inside the directory)
    and the tensors it places in them, as the reference's loader reads them
    (sardyne/loader/safetensors.py:110-131); otherwise every *.safetensors file of the directory,
    each name in one file only. Every header entry is checked against its file when the file is
    opened (SafeTensorsError)."""

    def __init__(self, directory):
        directory = pathlib.Path(directory)
        self.index = {}
        self._maps = []
        index = directory / "model.safetensors.index.json"
        if index.exists():
            try:
                weight_map = json.loads(index.read_text())["weight_map"]
            except (ValueError, KeyError, TypeError) as e:
                raise SafeTensorsError(f"{index.name}: no weight_map ({e})") from None
            if not isinstance(weight_map, dict):
                raise SafeTensorsError(f"{index.name}: weight_map is not an object")
            shards = {}
            for f in sorted(set(map(str, weight_map.values()))):
                # the index comes with the download: a shard is one path component of this
                # directory (no separators, no "." or ".."; symlinks, as in a hub cache, are fine)
                parts = pathlib.PurePath(f).parts
                if len(parts) != 1 or parts[0] in (".", "..") or pathlib.PurePath(f).suffix != ".safetensors":
                    raise SafeTensorsError(f"{index.name}: shard name {f!r} is not a file of the model directory")
                shards[f] = self._open(directory / f)
            for name, f in weight_map.items():
                if name not in shards[str(f)]:
                    raise SafeTensorsError(f"{index.name}: {name} placed in {f}, which does not hold it")
                self.index[name] = shards[str(f)][name]
        else:
            for path in sorted(directory.glob("*.safetensors")):
                for name, entry in self._open(path).items():
                    if name in self.index:
                        raise SafeTensorsError(f"{path.name}: {name} is also in another file")
                    self.index[name] = entry
        if not self.index:
            raise FileNotFoundError(f"no *.safetensors in {directory}")

    def _open(self, path) -> dict:
        """{name: (map, dtype, shape, begin, end)} of one file, every entry checked."""
        size = path.stat().st_size
        if size < 8:
            raise SafeTensorsError(f"{path.name}: {size} bytes, shorter than the header length")
        with open(path, "rb") as f:
            mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        (hlen,) = struct.unpack("<Q", mm[:8])
        if hlen > size - 8:  # checked before anything is read or allocated
            raise SafeTensorsError(f"{path.name}: header length {hlen} beyond the file")
        try:
            header = json.loads(mm[8:8 + hlen])
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise SafeTensorsError(f"{path.name}: header is not JSON ({e})") from None
        if not isinstance(header, dict):
            raise SafeTensorsError(f"{path.name}: header is not an object")
        base, out = 8 + hlen, {}
        for name, info in header.items():
            if name == "__metadata__":
                continue
            dtype, shape, b, e = _check_entry(f"{path.name}: {name}", info, size - base)
            out[name] = (mm, dtype, shape, base + b, base + e)
        self._maps.append(mm)
        return out

    def __contains__(self, name):
        return name in self.index

    def shape(self, name):
        return self.index[name][2]

    def get(self, name) -> np.ndarray:
        mm, dtype, shape, b, e = self.index[name]
        raw = np.frombuffer(mm, dtype=_ST_DTYPES[dtype], count=(e - b) // np.dtype(_ST_DTYPES[dtype]).itemsize,
                            offset=b)
        if dtype == "BF16":
            return (raw.astype(np.uint32) << 16).view(np.float32).reshape(shape)
        return raw.astype(np.float32).reshape(shape)


def rope_theta(cfg) -> float:
    """The RoPE base of config.json; scaled RoPE variants are refused (NotImplementedError: the
    engine runs plain RoPE), with the reference's config reader's rules
    (sardyne/loader/hf_config.py:12-27)."""
    given = cfg.get("rope_parameters") or {}
    # newer configs nest the parameters per attention kind; only full attention is supported
    per_kind = bool(given) and all(isinstance(v, dict) for v in given.values())
    if per_kind and "full_attention" not in given:
        raise NotImplementedError(f"RoPE parameters per layer kind {sorted(given)} are not supported")
    rope = given["full_attention"] if per_kind else given
    for source in (rope, cfg.get("rope_scaling") or {}):
        variant = source["rope_type"] if "rope_type" in source else source.get("type", "default")
        if variant is not None and variant != "default":
            raise NotImplementedError(f"RoPE scaling '{variant}' is not supported")
    return float(rope["rope_theta"] if "rope_theta" in rope else cfg.get("rope_theta", 10000.0))


def interleave_rope_rows(w: np.ndarray, n_head: int) -> np.ndarray:
    """HF rotates the two halves of each head; GGUF llama rotates adjacent pairs: within every head
    of rows [a0 .. a(h/2-1) | b0 .. b(h/2-1)] the order becomes a0 b0 a1 b1 ... (matrices and biases)."""
    rows = w.shape[0]
    half = rows // n_head // 2
    return w.reshape(n_head, 2, half, *w.shape[1:]).transpose(0, 2, 1, *range(3, w.ndim + 2)).reshape(w.shape)


def block_type(gguf_name: str, n_in: int, outtype: str, tied: bool) -> str:
    """The ggml type of a tensor: vectors, norms, biases and the router F32; matrices the requested
    type, with the fallbacks of the 32-element formats for rows that are not whole superblocks."""
    if gguf_name.endswith(("norm.weight", ".bias")) or "gate_inp" in gguf_name:
        return "F32"
    if outtype == "q4_k_m":
        return (synth.mix_q4_k_m_tied if tied else synth.mix_q4_k_m_untied)(gguf_name, n_in)
    kind = {"f32": "F32", "f16": "F16", "bf16": "BF16", "q8_0": "Q8_0", "q4_0": "Q4_0", "q4_k": "Q4_K",
            "q6_k": "Q6_K"}[outtype]
    if kind in kquant.QK and n_in % kquant.QK[kind]:
        kind = {"Q4_K": "Q5_0", "Q6_K": "Q8_0"}.get(kind, "F16") if n_in % 32 == 0 else "F16"
    return kind


F16_MAX = float(np.finfo(np.float16).max)


def encode(name: str, data: np.ndarray, kind: str):
    if kind == "F32":
        return np.ascontiguousarray(data, np.float32).view(np.uint8)
    if kind == "F16":
        # a value beyond the f16 range is refused rather than written as infinity, as the
        # reference's converter does (sardyne/loader/convert.py:97-101); the maximum of a tensor
        # holding a NaN is NaN, which passes, and its NaNs stay NaN
        peak = float(np.max(np.abs(data), initial=0.0))
        if peak > F16_MAX:
            raise ValueError(f"{name}: value {peak:g} beyond the f16 maximum ({F16_MAX:g}); use --outtype bf16")
        return np.ascontiguousarray(data, np.float16).view(np.uint8)
    if kind == "BF16":
        return f32_to_bf16(data).view(np.uint8)
    return np.frombuffer(kquant.quantize(data.reshape(-1, data.shape[-1]), kind), np.uint8)


def end_token_ids(hf_dir: pathlib.Path, cfg: dict) -> list:
    """The end-of-generation token ids: those of generation_config.json when it names any, else
    those of config.json (reference sardyne/loader/hf_config.py:30-42)."""
    gen = hf_dir / "generation_config.json"
    for source in (json.loads(gen.read_text()) if gen.exists() else {}, cfg):
        ids = source.get("eos_token_id")
        if ids is not None:
            return [int(i) for i in (ids if isinstance(ids, list) else [ids])]
    return []


def convert(hf_dir, out_path, outtype: str = "q4_k_m") -> pathlib.Path:
    hf_dir = pathlib.Path(hf_dir)
    cfg = json.loads((hf_dir / "config.json").read_text())
    arch = ARCHS.get((cfg.get("architectures") or [""])[0])
    if arch is None:
        raise NotImplementedError(f"architecture {cfg.get('architectures')} is not supported")
    if outtype not in FILE_TYPES:
        raise ValueError(f"outtype {outtype} is not one of {sorted(FILE_TYPES)}")
    st = SafeTensors(hf_dir)
    n_layer, dim = cfg["num_hidden_layers"], cfg["hidden_size"]
    n_head = cfg["num_attention_heads"]
    n_kv = cfg.get("num_key_value_heads", n_head)
    head_dim = cfg.get("head_dim") or dim // n_head
    tied = bool(cfg.get("tie_word_embeddings", False)) or "lm_head.weight" not in st
    moe = arch == "qwen3moe"

    w = GGUFWriter(out_path)
    meta = [("vocab_size", cfg["vocab_size"]), ("context_length", cfg.get("max_position_embeddings", 2048)),
            ("embedding_length", dim), ("block_count", n_layer), ("feed_forward_length", cfg["intermediate_size"]),
            ("attention.head_count", n_head), ("attention.head_count_kv", n_kv),
            ("rope.freq_base", rope_theta(cfg)), ("rope.dimension_count", head_dim),
            ("attention.layer_norm_rms_epsilon", float(cfg["rms_norm_eps"]))]
    if cfg.get("head_dim"):
        meta += [("attention.key_length", head_dim), ("attention.value_length", head_dim)]
    if moe:
        meta += [("expert_count", cfg["num_experts"]), ("expert_used_count", cfg["num_experts_per_tok"]),
                 ("expert_feed_forward_length", cfg["moe_intermediate_size"])]
    w.add("general.architecture", arch)
    w.add("general.name", hf_dir.name)
    for key, value in meta:
        w.add(f"{arch}.{key}", value)
    w.add("general.file_type", FILE_TYPES[outtype])
    if isinstance(cfg.get("bos_token_id"), int):  # a single id only
        w.add("tokenizer.ggml.bos_token_id", cfg["bos_token_id"])
    ends = end_token_ids(hf_dir, cfg)
    if ends:  # the first is the file's end-of-sequence token
        w.add("tokenizer.ggml.eos_token_id", ends[0])
    if (hf_dir / "tokenizer.json").exists():
        for key, value in tokenizer_fields(hf_dir, cfg["vocab_size"]).items():
            if key == "tokenizer.ggml.token_type":
                w.add(key, value, ARRAY, I32)
            elif isinstance(value, list):
                w.add(key, value, ARRAY, STRING)
            else:
                w.add(key, value)

    def add(gguf_name, shape, load):
        kind = block_type(gguf_name, shape[-1], outtype, tied)

        def produce(load=load, kind=kind, name=gguf_name):
            return encode(name, load(), kind).tobytes()

        w.add_lazy_tensor(gguf_name, tuple(reversed(shape)), kind, produce)

    def plain(hf_name, gguf_name, heads=None):
        def load():
            x = st.get(hf_name)
            return interleave_rope_rows(x, heads) if heads else x

        add(gguf_name, st.shape(hf_name), load)

    plain("model.embed_tokens.weight", "token_embd.weight")
    plain("model.norm.weight", "output_norm.weight")
    if not tied:
        plain("lm_head.weight", "output.weight")
    for i in range(n_layer):
        pre = f"model.layers.{i}."
        for hf, gg in LAYER_TENSORS:
            if pre + hf not in st:
                continue
            heads = None
            if arch == "llama" and gg.startswith(("attn_q.", "attn_k.")):
                heads = n_head if gg.startswith("attn_q.") else n_kv
            plain(pre + hf, f"blk.{i}.{gg}", heads)
        if moe:
            n_exp = cfg["num_experts"]
            for hf, gg in EXPERT_TENSORS:
                names = [f"{pre}mlp.experts.{e}.{hf}" for e in range(n_exp)]
                shape = (n_exp,) + st.shape(names[0])
                add(f"blk.{i}.{gg}", shape, lambda names=names: np.stack([st.get(n) for n in names]))
    return w.write()


def main():
    ap = argparse.ArgumentParser(description="Convert a Hugging Face checkpoint to GGUF (K-quants included)")
    ap.add_argument("hf_dir")
    ap.add_argument("out")
    ap.add_argument("--outtype", choices=sorted(FILE_TYPES), default="q4_k_m")
    args = ap.parse_args()
    print(convert(args.hf_dir, args.out, args.outtype))


if __name__ == "__main__":
    main()
