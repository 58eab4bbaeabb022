"""The decode step's fused kernels return exactly what the separate kernels return: the norm,
SwiGLU gate and activation quantization moved into the prologue of the consuming matvec, the
two-format projection launch (Q/K in Q4_K and V in Q6_K as one kernel), the MoE norm inside the
router and expert kernels, the whole MoE block as one kernel, and the L2 prefetch hints. Each configuration runs in its own process
(the switches are read once per process); logits must match bit for bit."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from sardyne_b200 import synth

pytestmark = pytest.mark.gpu

SPECS = {
    "dense-kquant": dict(arch="qwen2", dim=256, n_layer=3, head_dim=64, ffn=512, vocab=512, qkv_bias=True,
                         tied=False, std=0.02, kinds=synth.mix_q4_k_m_untied),
    "moe-kquant": dict(arch="qwen3moe", dim=256, n_layer=3, head_dim=64, n_expert=8, n_used=3, ffn_exp=256,
                       vocab=512, tied=False, qk_norm=True, std=0.02, kinds=synth.mix_q4_k_m_untied),
    # wide enough for the one-kernel MoE decode block (hidden size a multiple of 1024)
    "moe-block": dict(arch="qwen3moe", dim=1024, n_layer=3, n_head=8, n_kv_head=2, head_dim=128, n_expert=16,
                      n_used=4, ffn_exp=512, vocab=512, tied=False, qk_norm=True, std=0.02,
                      kinds=synth.mix_q4_k_m_untied),
}
PROMPT = [3, 14, 15, 9, 26, 5, 35, 8]
STEPS = 6

RUN = """
import json, sys, numpy as np
sys.path.insert(0, sys.argv[5])
import refruntime as rt
path, out, prompt, steps = sys.argv[1], sys.argv[2], json.loads(sys.argv[3]), int(sys.argv[4])
m = rt.model(path)
ctx = rt.Context(m, max_seq=64, n_batch=len(prompt))
logits = [ctx.eval(prompt)]
for i in range(steps):
    logits.append(ctx.eval([int(np.argmax(logits[-1])) + i % 3]))
np.save(out, np.stack(logits))
"""

CONFIGS = {
    "fused": {},
    "separate": {"SARDYNE_NO_FUSED_NORM": "1"},
    "moe-norm-fused": {"SARDYNE_MOE_NORM": "fused"},
    "no-prefetch": {"SARDYNE_L2_PREFETCH": "off"},
    "prefetch-all": {"SARDYNE_L2_PREFETCH": "all"},
    "no-graph": {"SARDYNE_NO_GRAPH": "1"},
    "moe-block-on": {"SARDYNE_MOE_DECODE": "on"},
}


def run(path, out, env_extra):
    env = dict(os.environ)
    for k in ("SARDYNE_NO_FUSED_NORM", "SARDYNE_MOE_NORM", "SARDYNE_L2_PREFETCH", "SARDYNE_NO_GRAPH",
              "SARDYNE_MOE_DECODE"):
        env.pop(k, None)
    env.update(env_extra)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env["PYTHONPATH"] = root + os.pathsep + env.get("PYTHONPATH", "")
    tests = os.path.dirname(os.path.abspath(__file__))
    r = subprocess.run([sys.executable, "-c", RUN, str(path), str(out), json.dumps(PROMPT), str(STEPS), tests], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return np.load(out)


@pytest.mark.parametrize("name", sorted(SPECS))
def test_fused_decode_matches_separate_kernels(tmp_path, name):
    path = tmp_path / "m.gguf"
    synth.write_model(path, synth.Spec(**SPECS[name], seed=5))
    got = {c: run(path, tmp_path / f"{c}.npy", env) for c, env in CONFIGS.items()}
    for c in CONFIGS:
        assert np.isfinite(got[c]).all(), c
        assert np.array_equal(got[c], got["separate"]), f"{c}: max diff {np.abs(got[c] - got['separate']).max()}"
