"""Weight quantizers (NumPy) for synthetic models: Q4_K, Q6_K, Q5_0, Q4_0, Q8_0.

The reference ships quantizers only for Q8_0 and Q4_0 (sardyne/quant.py:151-178); this module
adds its own simple min/max quantizers for the K-quants and Q5_0 so that N(0, 0.02) weights can
be turned into the block formats the hot path consumes. They target the byte layouts of the
reference (csrc/quant.h:16-43), not any particular third-party quantizer's choices: parity
never depends on them, because the GPU and the CPU oracle consume the same bytes.

  Q4_K  per 32-element sub-block: low = min(0, min x), step = (max x - low)/15; the superblock
        keeps f16 d = max step/63 and dmin = max(-low)/63, each sub-block 6-bit multiples of them,
        and q = round((x + dmin*m)/(d*sc)) clamped to 0..15.
  Q6_K  per 16-element group: step = max|x|/31; f16 d = max step/127, int8 sc = round(step/d),
        q = round(x/(d*sc)) clamped to -32..31.
  Q5_0  per 32: d = v/-16 where v is the signed largest-magnitude value, q = round(x/d) + 16
        clamped to 0..31 (the largest value lands exactly on q = 0).
  Q8_0  per 32: d = max|x|/127, q = round(x/d)   (as the reference, quant.py:151-163)
  Q4_0  per 32: d = v/-8, q = min(15, trunc(x/d + 8.5))  (as the reference, quant.py:165-178)
"""
import numpy as np

QK = {"Q8_0": 32, "Q4_0": 32, "Q5_0": 32, "Q4_K": 256, "Q6_K": 256}
BLOCK_BYTES = {"Q8_0": 34, "Q4_0": 18, "Q5_0": 22, "Q4_K": 144, "Q6_K": 210}


def _f16(v: np.ndarray) -> np.ndarray:
    return np.asarray(v, np.float32).astype(np.float16)


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return _f16(v).view(np.uint8).reshape(-1, 2)


def _safe_div(a, b):
    with np.errstate(divide="ignore", invalid="ignore"):
        return np.where(b != 0, a / np.where(b != 0, b, 1), 0).astype(np.float32)


def quantize_q4_k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, 8, 32)
    nb = x.shape[0]
    low = np.minimum(0.0, x.min(axis=2))                      # [nb, 8]
    step = (x.max(axis=2) - low) / np.float32(15)
    d = _f16(step.max(axis=1) / np.float32(63)).astype(np.float32)
    dmin = _f16((-low).max(axis=1) / np.float32(63)).astype(np.float32)
    sc = np.clip(np.rint(_safe_div(step, d[:, None])), 0, 63).astype(np.int32)
    m = np.clip(np.rint(_safe_div(-low, dmin[:, None])), 0, 63).astype(np.int32)
    eff_s = d[:, None] * sc
    eff_m = dmin[:, None] * m
    q = np.clip(np.rint(_safe_div(x + eff_m[:, :, None], eff_s[:, :, None])), 0, 15).astype(np.uint8)
    out = np.zeros((nb, 144), np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:4] = _f16_bytes(dmin)
    # 12-byte scale/min packing (decoded by csrc/quant.h:72-80)
    lo4, hi4 = sc[:, :4], sc[:, 4:]
    mlo4, mhi4 = m[:, :4], m[:, 4:]
    out[:, 4:8] = (lo4 | ((hi4 >> 4) << 6)).astype(np.uint8)
    out[:, 8:12] = (mlo4 | ((mhi4 >> 4) << 6)).astype(np.uint8)
    out[:, 12:16] = ((hi4 & 15) | ((mhi4 & 15) << 4)).astype(np.uint8)
    q = q.reshape(nb, 4, 2, 32)  # group g: sub-blocks 2g (low nibbles) and 2g+1 (high)
    out[:, 16:] = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(nb, 128)
    return out


def quantize_q6_k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, 16, 16)
    nb = x.shape[0]
    step = np.abs(x).max(axis=2) / np.float32(31)             # [nb, 16]
    d = _f16(step.max(axis=1) / np.float32(127)).astype(np.float32)
    sc = np.clip(np.rint(_safe_div(step, d[:, None])), -128, 127).astype(np.int32)
    eff = d[:, None] * sc
    q = np.clip(np.rint(_safe_div(x, eff[:, :, None])), -32, 31).astype(np.int32) + 32
    q = q.reshape(nb, 2, 4, 32).astype(np.uint8)               # [half][quarter][l]
    ql = np.empty((nb, 2, 64), np.uint8)
    ql[:, :, :32] = (q[:, :, 0] & 15) | ((q[:, :, 2] & 15) << 4)
    ql[:, :, 32:] = (q[:, :, 1] & 15) | ((q[:, :, 3] & 15) << 4)
    qh = (q[:, :, 0] >> 4) | ((q[:, :, 1] >> 4) << 2) | ((q[:, :, 2] >> 4) << 4) | ((q[:, :, 3] >> 4) << 6)
    out = np.zeros((nb, 210), np.uint8)
    out[:, 0:128] = ql.reshape(nb, 128)
    out[:, 128:192] = qh.reshape(nb, 64)
    out[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    out[:, 208:210] = _f16_bytes(d)
    return out


def _signed_max(x):
    idx = np.abs(x).argmax(axis=1)
    return x[np.arange(x.shape[0]), idx]


def quantize_q5_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, 32)
    d = _f16(_signed_max(x) / np.float32(-16)).astype(np.float32)
    q = np.clip(np.rint(_safe_div(x, d[:, None])) + 16, 0, 31).astype(np.uint32)
    out = np.zeros((x.shape[0], 22), np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    qh = ((q >> 4) & 1) << np.arange(32, dtype=np.uint32)
    out[:, 2:6] = qh.sum(axis=1, dtype=np.uint64).astype("<u4").view(np.uint8).reshape(-1, 4)
    out[:, 6:] = ((q[:, :16] & 15) | ((q[:, 16:] & 15) << 4)).astype(np.uint8)
    return out


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, 32)
    d = np.abs(x).max(axis=1) / np.float32(127)
    inv = _safe_div(np.float32(1), d)
    v = (x * inv[:, None]).astype(np.float64)
    q = (np.sign(v) * np.floor(np.abs(v) + 0.5)).astype(np.int8)  # roundf: half away from zero
    out = np.zeros((x.shape[0], 34), np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:] = q.view(np.uint8)
    return out


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).reshape(-1, 32)
    d = _signed_max(x) / np.float32(-8)
    inv = _safe_div(np.float32(1), d)
    q = np.minimum(15, np.trunc(x * inv[:, None] + np.float32(8.5)).astype(np.int32)).astype(np.uint8)
    out = np.zeros((x.shape[0], 18), np.uint8)
    out[:, 0:2] = _f16_bytes(d)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out


QUANTIZERS = {"Q4_K": quantize_q4_k, "Q6_K": quantize_q6_k, "Q5_0": quantize_q5_0, "Q8_0": quantize_q8_0,
              "Q4_0": quantize_q4_0}


def quantize(x: np.ndarray, kind: str, chunk_rows: int = 4096) -> bytes:
    """Quantize the rows of x ([..., n_in], n_in a multiple of the block) to `kind` bytes."""
    x = np.asarray(x, np.float32)
    n_in = x.shape[-1]
    if n_in % QK[kind]:
        raise ValueError(f"{kind}: row of {n_in} is not a multiple of {QK[kind]}")
    rows = x.reshape(-1, n_in)
    parts = [QUANTIZERS[kind](rows[i:i + chunk_rows]).reshape(-1) for i in range(0, rows.shape[0], chunk_rows)]
    return np.concatenate(parts).tobytes() if parts else b""


def synth_pool(kind: str, rng: np.random.Generator, std: float = 0.02, pool_blocks: int = 1 << 15) -> np.ndarray:
    """pool_blocks genuinely quantized blocks of N(0, std) values, [pool_blocks][block bytes]."""
    raw = quantize((rng.standard_normal((pool_blocks, QK[kind])) * std).astype(np.float32), kind)
    return np.frombuffer(raw, np.uint8).reshape(pool_blocks, BLOCK_BYTES[kind])


def synth_tensor(kind: str, n_rows: int, n_in: int, rng: np.random.Generator, std: float = 0.02,
                 pool_blocks: int = 1 << 15, pool: np.ndarray | None = None) -> bytes:
    """Bytes of an n_rows x n_in `kind` tensor that looks like quantized N(0, std) weights, made
    fast for multi-GB models: a pool of genuinely quantized blocks (drawn here, or `pool` shared
    by the tensors of one model) fills the tensor with blocks picked at random (every block is a
    real quantization of Gaussian values; only their arrangement is resampled)."""
    qk = QK[kind]
    n_blocks = n_rows * (n_in // qk)
    if pool is None and n_blocks <= pool_blocks:
        return quantize((rng.standard_normal((n_rows, n_in)) * std).astype(np.float32), kind)
    if pool is None:
        pool = synth_pool(kind, rng, std, pool_blocks)
    idx = rng.integers(0, len(pool), n_blocks)
    return pool[idx].tobytes()
