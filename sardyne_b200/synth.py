"""Synthetic GGUF models for tests and benchmarks (random init, reference tensor names).

``write_model(path, spec)`` writes a llama / qwen2 / qwen3 / qwen3moe GGUF with the metadata keys
the reference runtime reads (csrc/model_llama.c:225-319) and weights drawn from the spec's
distribution, each 2D/3D weight stored in the type spec.kind(name, n_in) picks.
"""
import dataclasses

import numpy as np

from . import kquant
from .gguf_writer import GGUFWriter, f32_to_bf16

ARCH_DEFAULTS = {"llama": {}, "qwen2": {}, "qwen3": {}, "qwen3moe": {}}


@dataclasses.dataclass
class Spec:
    arch: str = "llama"
    dim: int = 64
    n_layer: int = 2
    n_head: int = 4
    n_kv_head: int = 2
    head_dim: int = 16
    ffn: int = 128
    vocab: int = 64
    context: int = 64
    eps: float = 1e-5
    theta: float = 10000.0
    tied: bool = True
    qkv_bias: bool = False
    qk_norm: bool = False
    n_expert: int = 0
    n_used: int = 0
    ffn_exp: int = 0
    std: float = 0.0      # 0: N(0, 1/sqrt(n_in)) like the reference tests; else N(0, std)
    norm_noise: float = 0.1
    kinds: object = "F32"  # a type name, or a function (name, n_in) -> type name
    seed: int = 0
    synth: bool = False    # fill quantized tensors from one pool of quantized blocks per type (fast, multi-GB)

    def kind(self, name, n_in):
        k = self.kinds(name, n_in) if callable(self.kinds) else self.kinds
        if k in kquant.QK and n_in % kquant.QK[k]:
            raise ValueError(f"{name}: row {n_in} is not a multiple of the {k} block")
        return k


def q4_k_m(name, n_in, layer_parity=None):
    """The Q4_K_M-like mix of the BASELINE configs: Q4_K by default; Q6_K on attn_v, on the
    ffn_down (and ffn_down_exps) of even layers and on output (token_embd when tied); rows not
    a multiple of 256 fall back to Q5_0 (for Q4_K) and Q8_0 (for Q6_K); router, norms F32."""
    if "gate_inp" in name or name.endswith("norm.weight") or name.endswith(".bias"):
        return "F32"
    six = ("attn_v" in name or name in ("output.weight", "token_embd.weight") or
           ("ffn_down" in name and int(name.split(".")[1]) % 2 == 0))
    if n_in % 256:
        return "Q8_0" if six else "Q5_0"
    return "Q6_K" if six else "Q4_K"


def mix_q4_k_m_tied(name, n_in):
    return q4_k_m(name, n_in)


def mix_q4_k_m_untied(name, n_in):
    if name == "token_embd.weight":
        return "Q4_K" if n_in % 256 == 0 else "Q5_0"
    return q4_k_m(name, n_in)


def write_model(path, spec: Spec):
    rng = np.random.default_rng(spec.seed)
    s = spec
    w = GGUFWriter(path)
    a = s.arch
    w.add("general.architecture", a)
    w.add(f"{a}.vocab_size", s.vocab)
    w.add(f"{a}.context_length", s.context)
    w.add(f"{a}.embedding_length", s.dim)
    w.add(f"{a}.block_count", s.n_layer)
    w.add(f"{a}.feed_forward_length", s.ffn_exp * max(s.n_used, 1) if a == "qwen3moe" else s.ffn)
    w.add(f"{a}.attention.head_count", s.n_head)
    w.add(f"{a}.attention.head_count_kv", s.n_kv_head)
    w.add(f"{a}.attention.key_length", s.head_dim)
    w.add(f"{a}.attention.value_length", s.head_dim)
    w.add(f"{a}.rope.freq_base", float(s.theta))
    w.add(f"{a}.attention.layer_norm_rms_epsilon", float(s.eps))
    if a == "qwen3moe":
        w.add(f"{a}.expert_count", s.n_expert)
        w.add(f"{a}.expert_used_count", s.n_used)
        w.add(f"{a}.expert_feed_forward_length", s.ffn_exp)

    pools = {}  # synth: one pool of quantized blocks per type, shared by every tensor

    def tensor(name, *shape, vector=False, norm=False):
        n_in = shape[-1]
        if vector:
            v = (1 + rng.standard_normal(shape) * s.norm_noise) if norm else rng.standard_normal(shape) * 0.1
            w.add_tensor(name, v.astype(np.float32), "F32")
            return
        kind = s.kind(name, n_in)
        ne = tuple(reversed(shape))
        rows = int(np.prod(shape[:-1]))
        if kind in kquant.QK and s.synth:
            if kind not in pools:
                pools[kind] = kquant.synth_pool(kind, rng, s.std or 0.02)
            trng = np.random.default_rng([s.seed, len(w.tensors)])  # drawn when the file is written
            w.add_lazy_tensor(name, ne, kind,
                              lambda k=kind, r=rows, n=n_in, g=trng: kquant.synth_tensor(k, r, n, g, pool=pools[k]))
            return
        std = s.std or 1.0 / np.sqrt(n_in)
        data = (rng.standard_normal(shape) * std).astype(np.float32)
        if kind == "F32":
            w.add_tensor(name, data, "F32")
        elif kind == "F16":
            w.add_tensor(name, data, "F16")
        elif kind == "BF16":
            w.add_tensor(name, f32_to_bf16(data), "BF16")
        else:
            w.add_raw_tensor(name, ne, kind, kquant.quantize(data.reshape(-1, n_in), kind))

    q, kv = s.n_head * s.head_dim, s.n_kv_head * s.head_dim
    tensor("token_embd.weight", s.vocab, s.dim)
    tensor("output_norm.weight", s.dim, vector=True, norm=True)
    if not s.tied:
        tensor("output.weight", s.vocab, s.dim)
    for i in range(s.n_layer):
        p = f"blk.{i}."
        tensor(p + "attn_norm.weight", s.dim, vector=True, norm=True)
        tensor(p + "ffn_norm.weight", s.dim, vector=True, norm=True)
        tensor(p + "attn_q.weight", q, s.dim)
        tensor(p + "attn_k.weight", kv, s.dim)
        tensor(p + "attn_v.weight", kv, s.dim)
        tensor(p + "attn_output.weight", s.dim, q)
        if s.qkv_bias:
            tensor(p + "attn_q.bias", q, vector=True)
            tensor(p + "attn_k.bias", kv, vector=True)
            tensor(p + "attn_v.bias", kv, vector=True)
        if s.qk_norm:
            tensor(p + "attn_q_norm.weight", s.head_dim, vector=True, norm=True)
            tensor(p + "attn_k_norm.weight", s.head_dim, vector=True, norm=True)
        if a == "qwen3moe":
            tensor(p + "ffn_gate_inp.weight", s.n_expert, s.dim)
            tensor(p + "ffn_gate_exps.weight", s.n_expert, s.ffn_exp, s.dim)
            tensor(p + "ffn_up_exps.weight", s.n_expert, s.ffn_exp, s.dim)
            tensor(p + "ffn_down_exps.weight", s.n_expert, s.dim, s.ffn_exp)
        else:
            tensor(p + "ffn_gate.weight", s.ffn, s.dim)
            tensor(p + "ffn_up.weight", s.ffn, s.dim)
            tensor(p + "ffn_down.weight", s.dim, s.ffn)
    return w.write()


# The BASELINE model configurations (shapes from BASELINE.json configs 3-5).
SMOLLM2_135M = dict(arch="llama", dim=576, n_layer=30, n_head=9, n_kv_head=3, head_dim=64, ffn=1536, vocab=49152,
                    context=2048, eps=1e-5, theta=1e5, tied=True, std=0.02, kinds=mix_q4_k_m_tied)
QWEN25_3B = dict(arch="qwen2", dim=2048, n_layer=36, n_head=16, n_kv_head=2, head_dim=128, ffn=11008, vocab=151936,
                 context=4096, eps=1e-6, theta=1e6, tied=True, qkv_bias=True, std=0.02, kinds=mix_q4_k_m_tied)
QWEN3_30B_A3B = dict(arch="qwen3moe", dim=2048, n_layer=48, n_head=32, n_kv_head=4, head_dim=128, ffn=6144,
                     vocab=151936, context=4096, eps=1e-6, theta=1e6, tied=False, qk_norm=True, n_expert=128,
                     n_used=8, ffn_exp=768, std=0.02, kinds=mix_q4_k_m_untied)
BASELINE_MODELS = {"smollm2": SMOLLM2_135M, "qwen25_3b": QWEN25_3B, "qwen3moe": QWEN3_30B_A3B}
SYNTH_LAYOUT = 2  # bumped whenever the bytes write_model produces for a spec change


def model_cache_dir():
    """SARDYNE_MODEL_DIR, else /dev/shm when it has room for the largest model, else the temp dir."""
    import os
    import shutil
    import tempfile
    if os.environ.get("SARDYNE_MODEL_DIR"):
        return os.environ["SARDYNE_MODEL_DIR"]
    shm = "/dev/shm"
    try:
        if os.access(shm, os.W_OK) and shutil.disk_usage(shm).free > 24e9:
            return shm
    except OSError:
        pass
    return tempfile.gettempdir()


def baseline_model(name, directory=None, layers=0):
    """Path of the synthetic GGUF of a BASELINE config (3: smollm2, 4: qwen25_3b, 5: qwen3moe),
    written once (quantized blocks from one pool per type, seed 0) and reused from the cache.
    layers > 0: the same shape with only that many layers (small cases for profiling)."""
    import os
    import pathlib
    cut = f"-L{layers}" if layers else ""
    path = pathlib.Path(directory or model_cache_dir()) / f"sardyne-{name}{cut}-v{SYNTH_LAYOUT}.gguf"
    if not path.exists():
        spec = dict(BASELINE_MODELS[name], **({"n_layer": layers} if layers else {}))
        write_model(path, Spec(**spec, synth=True, seed=0))
        os.chmod(path, 0o644)
    return path
