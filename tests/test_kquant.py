"""The package's weight quantizers produce valid blocks with small error (checked by the oracle)."""
import numpy as np
import pytest

import oracle
from sardyne_b200 import kquant

# Relative RMS error bounds the reference accepts for published Q4_K_M files (tests/test_quant.py:53).
LIMITS = {"Q8_0": 0.01, "Q6_K": 0.03, "Q5_0": 0.07, "Q4_K": 0.11, "Q4_0": 0.15}


@pytest.mark.parametrize("kind", sorted(LIMITS))
def test_quantizer_error(kind):
    x = (np.random.default_rng(0).standard_normal((16, 512)) * 0.02).astype(np.float32)
    raw = np.frombuffer(kquant.quantize(x, kind), np.uint8)
    assert raw.size == 16 * 512 // kquant.QK[kind] * kquant.BLOCK_BYTES[kind]
    deq = oracle.dequant(raw, kind, 512)
    rel = np.sqrt(np.mean((deq - x) ** 2) / np.mean(x ** 2))
    assert rel < LIMITS[kind], rel


def test_q8_0_and_q4_0_match_reference_quantizer_bytes():
    """The two formats the reference can quantize: same bytes as its quantizer (via the golden
    activation vectors, whose Q8_0 bytes come from the reference C code)."""
    import pathlib
    g = np.load(pathlib.Path(__file__).parent / "golden" / "quant_golden.npz")
    assert kquant.quantize(g["act_x"], "Q8_0") == g["act_Q8_0"].tobytes()


def test_synth_tensor_blocks_are_valid():
    rng = np.random.default_rng(1)
    raw = np.frombuffer(kquant.synth_tensor("Q6_K", 300, 512, rng, pool_blocks=64), np.uint8)
    assert raw.size == 300 * 2 * 210
    deq = oracle.dequant(raw, "Q6_K", 512)
    assert np.isfinite(deq).all() and 0.01 < deq.std() < 0.03
