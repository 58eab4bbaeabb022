"""The GPU engine (engine_* C-ABI) against the reference engine on the same synthetic GGUFs.

The reference side is the reference's own libsardyne built from its sources (oracle/_ref), run
on the CPU with its scalar kernels. Both are driven by the reference's own, unmodified Python
runtime (sardyne.runtime through sardyne.capi, with SARDYNE_LIB naming the library), which is the
drop-in claim. The quantized products agree bit for bit; RMSNorm, RoPE, softmax and attention run
in fp32 on both sides in different summation orders, so logits are compared with a tolerance
proportional to their scale, plus greedy-token identity. Mirrors the reference's
tests/test_runtime.py:160-284 and tests/test_moe.py:286-435.
"""
import numpy as np
import pytest

import oracle
import refruntime as rt
from refruntime import Context, generate
from sardyne_b200 import synth
from sardyne_b200.gguf_writer import GGUFWriter

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")]

TOKENS = [3, 14, 15, 9, 26, 5, 35, 8, 2, 7, 1, 60]

SPECS = {
    "llama-f32": dict(),
    "llama-f16": dict(kinds="F16"),
    "llama-q8_0": dict(kinds="Q8_0"),
    "llama-q4_0": dict(kinds="Q4_0"),
    "llama-bias-q8_0": dict(qkv_bias=True, tied=False, kinds="Q8_0"),
    "qwen2-q4_0": dict(arch="qwen2", tied=False, qkv_bias=True, kinds="Q4_0"),
    "qwen3-bf16": dict(arch="qwen3", qk_norm=True, kinds="BF16"),
    "qwen3-q8_0": dict(arch="qwen3", qk_norm=True, kinds="Q8_0"),
    "kquant-mix": dict(dim=256, head_dim=64, ffn=512, tied=False, kinds=synth.mix_q4_k_m_untied),
    "kquant-q6k": dict(arch="qwen2", dim=256, head_dim=64, ffn=512, qkv_bias=True, kinds="Q6_K"),
    "smol-mix": dict(dim=576, n_head=9, n_kv_head=3, head_dim=64, ffn=1536, vocab=512, std=0.02,
                     kinds=synth.mix_q4_k_m_tied),
    "moe-f32": dict(arch="qwen3moe", dim=32, head_dim=16, n_expert=8, n_used=3, ffn_exp=64, tied=False, qk_norm=True),
    "moe-bf16": dict(arch="qwen3moe", dim=32, head_dim=16, n_expert=8, n_used=3, ffn_exp=64, tied=False,
                     qk_norm=True, kinds="BF16"),
    "moe-q8_0-128x8": dict(arch="qwen3moe", dim=32, head_dim=16, n_expert=128, n_used=8, ffn_exp=64, tied=False,
                           qk_norm=True, kinds="Q8_0"),
    "moe-one": dict(arch="qwen3moe", dim=32, head_dim=16, n_expert=1, n_used=1, ffn_exp=64, tied=False, qk_norm=True),
    "moe-kquant": dict(arch="qwen3moe", dim=256, head_dim=64, n_expert=8, n_used=3, ffn_exp=256, tied=False,
                       qk_norm=True, kinds=synth.mix_q4_k_m_untied),
    # single-token steps take the one-kernel MoE block (hidden size a multiple of 1024)
    "moe-block": dict(arch="qwen3moe", dim=1024, n_head=8, n_kv_head=2, head_dim=128, n_expert=16, n_used=4,
                      ffn_exp=512, vocab=512, tied=False, qk_norm=True, std=0.02, kinds=synth.mix_q4_k_m_untied),
    # a float router wider than the fused router kernel's shared memory: the generic matmul,
    # softmax and top-k kernels
    "moe-wide-router": dict(arch="qwen3moe", dim=6144, n_layer=1, n_head=4, n_kv_head=2, head_dim=64, n_expert=8,
                            n_used=2, ffn_exp=256, vocab=256, tied=False, qk_norm=True, std=0.02,
                            kinds=lambda name, n_in: "F32" if "gate_inp" in name or "norm" in name else "Q8_0"),
}


@pytest.fixture(scope="module", params=sorted(SPECS))
def model_path(request, tmp_path_factory):
    path = tmp_path_factory.mktemp(request.param) / "m.gguf"
    synth.write_model(path, synth.Spec(**{"context": 128, **SPECS[request.param]}, seed=len(request.param)))
    return path


@pytest.fixture(scope="module")
def ref_lib():
    """The reference library's path; its scalar kernels (the order the GPU products reproduce
    bit for bit) are selected for the module."""
    lib = oracle.ref()
    lib.op_set_simd(0)
    yield oracle.REF_LIB
    lib.op_set_simd(1)


def Model(path, lib=None):
    return rt.model(path, lib)


def close(got, want, scale=1e-3):
    tol = scale * max(1.0, float(np.abs(want).max()))
    assert np.abs(got - want).max() <= tol, (float(np.abs(got - want).max()), tol)


def test_forward_matches_reference(model_path, ref_lib):
    want = Context(Model(model_path, ref_lib), max_seq=32, n_batch=len(TOKENS),
                           logits_all=True).eval(TOKENS)
    got = Context(Model(model_path), max_seq=32, n_batch=len(TOKENS), logits_all=True).eval(TOKENS)
    close(got, want)
    assert (got.argmax(-1) == want.argmax(-1)).all()


LONG = [(7 * i + 3) % 60 + 1 for i in range(45)]


@pytest.mark.parametrize("n_batch", [45, 20])
def test_long_prompt_matches_reference(model_path, ref_lib, n_batch):
    """A 45-token prompt in one chunk or in chunks of 20 (the second and third start at positions
    20 and 40): the tensor-core GEMM and the query-tile prefill attention."""
    want = Context(Model(model_path, ref_lib), max_seq=64, n_batch=n_batch,
                           logits_all=True).eval(LONG)
    got = Context(Model(model_path), max_seq=64, n_batch=n_batch, logits_all=True).eval(LONG)
    close(got, want)
    assert (got.argmax(-1) == want.argmax(-1)).all()


def test_generate_matches_reference(model_path, ref_lib):
    """64 greedy steps (the reference's greedy loop, sardyne/runtime.py:115-140)."""
    want = generate(Context(Model(model_path, ref_lib), max_seq=80), TOKENS[:4], 64)
    got = generate(Context(Model(model_path), max_seq=80), TOKENS[:4], 64)
    assert len(want) == 64 and got == want


def test_info_matches_reference(model_path, ref_lib):
    a, b = Model(model_path).info, Model(model_path, ref_lib).info
    assert bytes(a) == bytes(b)


def test_kv_cache_and_batching(model_path):
    model = Model(model_path)
    full = Context(model, max_seq=32, n_batch=len(TOKENS), logits_all=True).eval(TOKENS)
    chunked = Context(model, max_seq=32, n_batch=5, logits_all=True).eval(TOKENS)
    close(chunked, full, 1e-4)
    ctx = Context(model, max_seq=32, n_batch=4)
    close(ctx.eval(TOKENS[:7]), full[6], 1e-4)
    for i, t in enumerate(TOKENS[7:], start=7):
        close(ctx.eval([t]), full[i], 1e-4)
    assert ctx.n_past == len(TOKENS)
    ctx.reset()
    assert ctx.n_past == 0
    close(ctx.eval(TOKENS), full[-1], 1e-4)


def test_truncate(model_path):
    model = Model(model_path)
    full = Context(model, max_seq=32, n_batch=len(TOKENS), logits_all=True).eval(TOKENS)
    ctx = Context(model, max_seq=32, n_batch=4)
    ctx.eval(TOKENS[:7])
    ctx.truncate(3)
    assert ctx.n_past == 3
    ctx.eval([60, 61])
    ctx.truncate(3)
    close(ctx.eval(TOKENS[3:]), full[-1], 1e-4)
    for bad in (-1, len(TOKENS) + 1):
        with pytest.raises(ValueError, match="posizione"):
            ctx.truncate(bad)
        assert ctx.n_past == len(TOKENS)


def test_results_are_deterministic(model_path):
    model = Model(model_path)
    outs = []
    for n_threads in (0, 1, 7):
        ctx = Context(model, max_seq=32, n_batch=len(TOKENS), logits_all=True, n_threads=n_threads)
        assert ctx.n_threads == n_threads
        outs.append(np.concatenate([ctx.eval(TOKENS[:8]), ctx.eval(TOKENS[8:])]))
    for o in outs[1:]:
        assert np.array_equal(o, outs[0])


def test_errors_leave_context_unchanged(tmp_path):
    path = synth.write_model(tmp_path / "m.gguf", synth.Spec(context=8))
    model = Model(path)
    ctx = Context(model, max_seq=8, n_batch=4)
    ctx.eval([1, 2, 3])
    for bad, msg in [([1] * 6, "contesto pieno"), ([64], "vocabolario"), ([-1], "vocabolario"), ([], "nessun")]:
        with pytest.raises(ValueError, match=msg):
            ctx.eval(bad)
        assert ctx.n_past == 3
    with pytest.raises(ValueError, match="n_batch"):
        Context(model, max_seq=8, n_batch=0)
    with pytest.raises(ValueError, match="max_seq"):
        Context(model, max_seq=0)
    with pytest.raises(ValueError, match="n_threads"):
        Context(model, max_seq=8, n_threads=-1)
    all_ctx = Context(model, max_seq=8, n_batch=2, logits_all=True)
    assert all_ctx.eval([1, 2, 3, 4, 5]).shape == (5, model.info.n_vocab)


def test_load_errors(tmp_path):
    with pytest.raises(ValueError, match="impossibile aprire"):
        Model(tmp_path / "missing.gguf")
    for n_expert, n_used, msg in [(0, 3, "expert_count"), (8, 0, "expert_used_count"), (8, 9, "expert_used_count")]:
        p = tmp_path / f"e{n_expert}_{n_used}.gguf"
        w = GGUFWriter(p)
        w.add("general.architecture", "qwen3moe")
        for k, v in [("embedding_length", 32), ("block_count", 1), ("feed_forward_length", 64),
                     ("attention.head_count", 2)]:
            w.add(f"qwen3moe.{k}", v)
        if n_expert:
            w.add("qwen3moe.expert_count", n_expert)
        w.add("qwen3moe.expert_used_count", n_used)
        w.add_tensor("token_embd.weight", np.zeros((8, 32), np.float32))
        w.write()
        with pytest.raises(ValueError, match=msg):
            Model(p)


def rewrite_gguf(src, dst, tensor_fn):
    """Copy a GGUF written by synth (U32 / F32 / string metadata) with every tensor passed through
    tensor_fn(name, ne, type_name, raw) -> (type_name, raw)."""
    import ctypes
    from sardyne_b200 import capi
    lib = capi.lib()
    err = ctypes.create_string_buffer(256)
    h = lib.gguf_open(str(src).encode(), err, len(err))
    assert h, err.value
    w = GGUFWriter(dst)
    try:
        for i in range(lib.gguf_n_kv(h)):
            kv = lib.gguf_get_kv(h, i).contents
            key = kv.key.decode()
            if kv.type == 8:
                n = ctypes.c_uint64()
                p = lib.gguf_kv_get_str(h, i, ctypes.byref(n))
                w.add(key, ctypes.string_at(p, n.value).decode())
            elif kv.type == 6:
                w.add(key, ctypes.c_float.from_address(kv.ptr).value, 6)
            else:
                w.add(key, ctypes.c_uint32.from_address(kv.ptr).value, 4)
        for i in range(lib.gguf_n_tensors(h)):
            t = lib.gguf_get_tensor(h, i).contents
            ne = tuple(t.ne[:t.n_dims])
            kind, raw = tensor_fn(t.name.decode(), ne, lib.gguf_type_name(t.type).decode(),
                                  ctypes.string_at(t.data, t.nbytes))
            w.add_raw_tensor(t.name.decode(), ne, kind, raw)
    finally:
        lib.gguf_close(h)
    return w.write()


def test_unsupported_tensors_are_rejected(tmp_path):
    """A Q4_1 matrix (a type the runtime does not run) is rejected by name and type."""
    src = synth.write_model(tmp_path / "src.gguf", synth.Spec())

    def q41(name, ne, kind, raw):
        if name == "blk.0.attn_q.weight":
            return "Q4_1", bytes(int(np.prod(ne)) // 32 * 20)
        return kind, raw

    with pytest.raises(ValueError, match="Q4_1 non supportato"):
        Model(rewrite_gguf(src, tmp_path / "q41.gguf", q41))


def test_moe_ties_choose_the_lowest_experts(tmp_path, ref_lib):
    """Router weights all zero: equal probabilities, the first k experts win (as the reference)."""
    src = synth.write_model(tmp_path / "src.gguf", synth.Spec(**SPECS["moe-f32"]))

    def zero_router(name, ne, kind, raw):
        return kind, (bytes(len(raw)) if "gate_inp" in name else raw)

    path = rewrite_gguf(src, tmp_path / "ties.gguf", zero_router)
    want = Context(Model(path, ref_lib), max_seq=32, n_batch=len(TOKENS),
                           logits_all=True).eval(TOKENS)
    got = Context(Model(path), max_seq=32, n_batch=len(TOKENS), logits_all=True).eval(TOKENS)
    close(got, want)


def greedy_on_device(ctx, tokens):
    """sdy_engine_eval_greedy through the C-ABI on a reference-runtime Context's handle."""
    import ctypes
    from sardyne_b200 import capi
    arr = (ctypes.c_int32 * len(tokens))(*tokens)
    nxt = ctypes.c_int32(-1)
    assert capi.lib().sdy_engine_eval_greedy(ctx._h, arr, len(tokens), ctypes.byref(nxt)) == 0, \
        capi.lib().engine_last_error(ctx._h)
    return nxt.value


def test_greedy_on_device_matches_host_argmax(model_path):
    """The device's greedy choice equals numpy.argmax of engine_eval's logits, step by step."""
    model = Model(model_path)
    host, dev = Context(model, max_seq=48, n_batch=8), Context(model, max_seq=48, n_batch=8)
    want = int(np.argmax(host.eval(TOKENS[:5])))
    got = greedy_on_device(dev, TOKENS[:5])
    for _ in range(24):
        assert got == want
        want = int(np.argmax(host.eval([want])))
        got = greedy_on_device(dev, [got])
    assert dev.n_past == host.n_past


def test_greedy_on_device_ties_take_the_lowest_id(tmp_path):
    """All logits equal (zero embeddings): the first id, as numpy.argmax."""
    src = synth.write_model(tmp_path / "src.gguf", synth.Spec())

    def zero_embd(name, ne, kind, raw):
        return kind, (bytes(len(raw)) if name == "token_embd.weight" else raw)

    model = Model(rewrite_gguf(src, tmp_path / "zero.gguf", zero_embd))
    ctx = Context(model, max_seq=16, n_batch=4)
    assert greedy_on_device(ctx, [3, 5]) == 0
    assert not ctx.eval([7]).any()  # the logits themselves are all zero
