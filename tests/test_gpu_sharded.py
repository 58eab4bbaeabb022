"""The sharded engine on 2 GPUs (one process each, NCCL all-reduce) returns the one-GPU logits bit
for bit: attention heads (with their KV cache and the attention-output rows), dense FFN rows and
MoE experts split across the ranks, prefill through the tensor-core GEMM and single-token steps
replayed from CUDA graphs; on small models and at the BASELINE Qwen2.5-3B and Qwen3-30B-A3B shapes
(whose one-GPU logits equal the reference engine's, tests/test_gpu_baseline_shapes.py). Needs two
GPUs; skipped otherwise."""
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
}
PROMPT = list(range(3, 43))  # 40 tokens: the prefill products go through the GEMM
STEPS = 5


def run_model(path):
    import refruntime as rt
    m = rt.model(str(path))
    ctx = rt.Context(m, max_seq=96, n_batch=len(PROMPT))
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


def _rank(rank, world, port, path, q):
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from sardyne_b200 import runtime
        runtime.shard_from_torch()
        q.put((rank, run_model(path)))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name", sorted(SPECS) + ["qwen25_3b", "qwen3moe"])
def test_two_ranks_match_one_gpu(tmp_path, name):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    if name in SPECS:
        path = tmp_path / f"{name}.gguf"
        synth.write_model(path, synth.Spec(**SPECS[name], seed=11))
    else:
        path = synth.baseline_model(name)
    want = run_model(path)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, str(path), q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(60)
    for r in range(2):
        assert not isinstance(got[r], str), got[r]
        assert np.array_equal(got[r], want), f"rank {r}: max diff {np.abs(got[r] - want).max()}"
