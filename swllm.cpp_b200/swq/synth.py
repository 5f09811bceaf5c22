"""Seeded synthetic GGUF weight blocks and activations.

The generators follow the published benchmark shapes' value distributions:
per-block ``d = fp16(|N(0,1)| * 2e-3)`` and ``dmin = fp16(|N(0,1)| * 1e-3)``,
6-bit K-quant scales/mins uniform over 0..63 (uniform random bytes in the
12-byte field decode to exactly that through get_scale_min_k4,
src/tensor.h:218-227), Q6_K int8 scales and Q3_K packed scales uniform over
their code range, quant bits uniform, Q8_0 int8 values uniform in -127..127,
activations fp32 N(0,1).

Block layouts are the GGUF ones read by the reference (src/tensor.h:136-432,
sizes src/gguf.h:60-86); a matrix is N rows of K/QK consecutive blocks.
"""
from __future__ import annotations

import numpy as np

Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 2, 8, 10, 11, 12, 13, 14

# type id -> (elements per block, bytes per block, offset of d, offset of dmin or None)
LAYOUT = {
    Q4_0: (32, 18, 0, None),
    Q8_0: (32, 34, 0, None),
    Q2_K: (256, 84, 80, 82),
    Q3_K: (256, 110, 108, None),
    Q4_K: (256, 144, 0, 2),
    Q5_K: (256, 176, 0, 2),
    Q6_K: (256, 210, 208, None),
}
NAMES = {Q4_0: "Q4_0", Q8_0: "Q8_0", Q2_K: "Q2_K", Q3_K: "Q3_K",
         Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
IDS = {v: k for k, v in NAMES.items()}


def block_geometry(type_id: int) -> tuple[int, int]:
    qk, bb, _, _ = LAYOUT[type_id]
    return qk, bb


def row_bytes(type_id: int, K: int) -> int:
    qk, bb = block_geometry(type_id)
    if K % qk:
        raise ValueError(f"K={K} is not a multiple of {qk}")
    return (K // qk) * bb


def matrix_bytes(type_id: int, N: int, K: int) -> int:
    return N * row_bytes(type_id, K)


def _half_bytes(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(v.shape + (2,))


def random_blocks(type_id: int, N: int, K: int, seed: int = 0,
                  d_scale: float = 2e-3, dmin_scale: float = 1e-3) -> np.ndarray:
    """Return a uint8 array [N, row_bytes] of seeded random blocks."""
    qk, bb, d_off, m_off = LAYOUT[type_id]
    nb = K // qk
    if nb * qk != K:
        raise ValueError(f"K={K} is not a multiple of {qk}")
    rng = np.random.default_rng(seed)
    blk = rng.integers(0, 256, size=(N, nb, bb), dtype=np.uint8)
    if type_id == Q8_0:
        blk[:, :, 2:] = rng.integers(-127, 128, size=(N, nb, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    d = np.abs(rng.standard_normal((N, nb), dtype=np.float32)) * np.float32(d_scale)
    blk[:, :, d_off:d_off + 2] = _half_bytes(d)
    if m_off is not None:
        dm = np.abs(rng.standard_normal((N, nb), dtype=np.float32)) * np.float32(dmin_scale)
        blk[:, :, m_off:m_off + 2] = _half_bytes(dm)
    return blk.reshape(N, nb * bb)


def fast_random_blocks(type_id: int, N: int, K: int, seed: int = 0,
                       d_scale: float = 2e-3, dmin_scale: float = 1e-3) -> np.ndarray:
    """random_blocks' value distributions drawn from 64-bit words (about 3
    GB/s), for model-sized matrices; the bytes differ from random_blocks' for
    the same seed.  Q8_0 quants stay in -127..127."""
    qk, bb, d_off, m_off = LAYOUT[type_id]
    nb = K // qk
    if nb * qk != K:
        raise ValueError(f"K={K} is not a multiple of {qk}")
    rng = np.random.default_rng(seed)
    n = N * nb * bb
    words = rng.integers(0, 2 ** 64, size=(n + 7) // 8, dtype=np.uint64)
    blk = words.view(np.uint8)[:n].reshape(N, nb, bb)
    if type_id == Q8_0:
        q = blk[:, :, 2:]
        q[q == 0x80] = 0x81
    d = np.abs(rng.standard_normal((N, nb), dtype=np.float32)) * np.float32(d_scale)
    blk[:, :, d_off:d_off + 2] = _half_bytes(d)
    if m_off is not None:
        dm = np.abs(rng.standard_normal((N, nb), dtype=np.float32)) * np.float32(dmin_scale)
        blk[:, :, m_off:m_off + 2] = _half_bytes(dm)
    return blk.reshape(N, nb * bb)


def random_activations(M: int, K: int, seed: int = 1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((M, K), dtype=np.float32)


def set_block_scale(blocks: np.ndarray, type_id: int, half_bits: int, which: str = "d",
                    row: int = 0, block: int = 0) -> None:
    """Overwrite one block's fp16 d (or dmin) with raw half bits (edge cases)."""
    qk, bb, d_off, m_off = LAYOUT[type_id]
    off = d_off if which == "d" else m_off
    if off is None:
        raise ValueError(f"{NAMES[type_id]} has no {which}")
    base = block * bb + off
    blocks[row, base] = half_bits & 0xFF
    blocks[row, base + 1] = (half_bits >> 8) & 0xFF
