"""The sharded engine on 2 GPUs (one process each) returns the one-GPU logits bit for bit:
attention heads (with their KV cache and the attention-output rows), dense FFN rows and MoE
experts split across the ranks, prefill through the tensor-core GEMM and single-token steps
replayed from CUDA graphs; on small models and at the BASELINE Qwen2.5-3B and Qwen3-30B-A3B shapes
(whose one-GPU logits equal the reference engine's, tests/test_gpu_baseline_shapes.py). The
exchanges go over NVLink peer memory (single-token sizes) and NCCL (prefill), and all over NCCL
with SARDYNE_EXCHANGE=nccl. "dense-kv1" has one KV head, so the two ranks share it (each holds
half of the query heads), and a vocabulary that is not a multiple of 4 (the exchange's scalar
copy). Needs two GPUs; skipped otherwise."""
import os
import socket

import numpy as np
import pytest

from sardyne_b200 import synth

pytestmark = pytest.mark.gpu

SPECS = {
    "dense": dict(arch="qwen2", dim=256, n_layer=2, n_head=4, n_kv_head=2, head_dim=64, ffn=512, vocab=1024,
                  context=128, qkv_bias=True, tied=True, std=0.02, kinds=synth.mix_q4_k_m_tied),
    "moe": dict(arch="qwen3moe", dim=256, n_layer=2, n_head=4, n_kv_head=2, head_dim=64, ffn=512, vocab=1024,
                context=128, qk_norm=True, tied=False, n_expert=8, n_used=2, ffn_exp=256, std=0.02,
                kinds=synth.mix_q4_k_m_untied),
    "dense-kv1": dict(arch="llama", dim=256, n_layer=2, n_head=4, n_kv_head=1, head_dim=64, ffn=512, vocab=1003,
                      context=128, tied=True, std=0.02, kinds=synth.mix_q4_k_m_tied),
}
PROMPT = list(range(3, 43))  # 40 tokens: the prefill products go through the GEMM
STEPS = 5


def run_model(path, exchange=None):
    """Logits of the prompt and STEPS single-token steps; with `exchange`, the context's exchange
    kind (sdy_engine_exchange) must be that."""
    import refruntime as rt
    m = rt.model(str(path))
    ctx = rt.Context(m, max_seq=96, n_batch=len(PROMPT))
    if exchange is not None:
        from sardyne_b200 import capi
        assert capi.lib().sdy_engine_exchange(ctx._h) == exchange
    if m.info.n_vocab > 100000:  # BASELINE shapes: prompt ids spread over the vocabulary
        prompt = np.random.default_rng(0).integers(0, m.info.n_vocab, len(PROMPT)).tolist()
        out = [ctx.eval(prompt)]
        for i in range(STEPS):
            out.append(ctx.eval([int(np.argmax(out[-1]))]))
        return np.stack(out)
    out = [ctx.eval(PROMPT)]
    for i in range(STEPS):
        out.append(ctx.eval([int(np.argmax(out[-1])) + i % 2]))
    return np.stack(out)


def _rank(rank, world, port, path, mode, q):
    import torch
    import torch.distributed as dist
    if mode == "nccl":
        os.environ["SARDYNE_EXCHANGE"] = "nccl"
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from sardyne_b200 import runtime
        runtime.shard_from_torch()
        q.put((rank, run_model(path, exchange=0 if mode == "nccl" else 1)))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _model(tmp_path, name):
    if name in SPECS:
        path = tmp_path / f"{name}.gguf"
        synth.write_model(path, synth.Spec(**SPECS[name], seed=11))
        return path
    return synth.baseline_model(name)


def _compare(path, world, mode):
    import torch.multiprocessing as mp
    want = run_model(path)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, str(path), mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(60)
    for r in range(world):
        assert not isinstance(got[r], str), got[r]
        assert np.array_equal(got[r], want), f"rank {r}: max diff {np.abs(got[r] - want).max()}"


@pytest.mark.parametrize("name,mode", [(n, m) for n in sorted(SPECS) for m in ("peer", "nccl")] +
                         [("qwen25_3b", "peer"), ("qwen3moe", "peer")])
def test_two_ranks_match_one_gpu(tmp_path, name, mode):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _compare(_model(tmp_path, name), 2, mode)


@pytest.mark.parametrize("name", sorted(SPECS) + ["qwen3moe"])
def test_every_gpu_matches_one_gpu(tmp_path, name):
    """On every GPU of the box (4 or 8): at 8 the Qwen3-30B-A3B shape holds 16 experts per rank and
    two ranks share each KV head; the small models' 4 query heads do not split 8 ways, so their
    attention stays replicated there."""
    import torch
    world = torch.cuda.device_count()
    if world < 4:
        pytest.skip("needs four or more GPUs")
    _compare(_model(tmp_path, name), min(world, 8), "peer")
