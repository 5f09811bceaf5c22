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


def _k4_unpack(s: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """[..., 12] packed K-quant scale bytes -> (scales, mins) [..., 8]
    (get_scale_min_k4, src/tensor.h:218-227)."""
    s = s.astype(np.int32)
    sc = np.empty(s.shape[:-1] + (8,), np.int32)
    mn = np.empty_like(sc)
    for j in range(4):
        sc[..., j] = s[..., j] & 63
        mn[..., j] = s[..., j + 4] & 63
        sc[..., j + 4] = (s[..., j + 8] & 15) | ((s[..., j] >> 6) << 4)
        mn[..., j + 4] = (s[..., j + 8] >> 4) | ((s[..., j + 4] >> 6) << 4)
    return sc, mn


def _k4_pack(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    out = np.empty(sc.shape[:-1] + (12,), np.int32)
    for j in range(4):
        out[..., j] = (sc[..., j] & 63) | ((sc[..., j + 4] >> 4) << 6)
        out[..., j + 4] = (mn[..., j] & 63) | ((mn[..., j + 4] >> 4) << 6)
        out[..., j + 8] = (sc[..., j + 4] & 15) | ((mn[..., j + 4] & 15) << 4)
    return out.astype(np.uint8)


def centred_blocks(type_id: int, N: int, K: int, seed: int = 0, d_scale: float = 2e-3) -> np.ndarray:
    """random_blocks with the mins of the formats that have them (Q2_K, Q4_K,
    Q5_K) chosen as a quantizer chooses them: each sub-block's values centred
    on zero (dmin per block, min codes = round(mean of d * scale * q / dmin)).
    The other formats are centred by construction (zero point in the middle of
    the code range) and come back as random_blocks.  Benchmark-distribution
    blocks (independent uniform min codes) give every Q4_K weight a mean of
    about +0.45, and a random model built of them amplifies rounding by orders
    of magnitude; a quantized real model does not."""
    blk = random_blocks(type_id, N, K, seed, d_scale=d_scale)
    if type_id not in (Q2_K, Q4_K, Q5_K):
        return blk
    qk, bb, d_off, m_off = LAYOUT[type_id]
    b = blk.reshape(N, K // qk, bb)
    d = b[..., d_off:d_off + 2].copy().view(np.float16)[..., 0].astype(np.float64)
    if type_id == Q2_K:
        sc = (b[..., :16] & 15).astype(np.int32)
        target = 1.5 * d[..., None] * sc                       # mean of d * sc * q, q uniform 0..3
        dmin = (target.max(axis=-1) / 15.0).astype(np.float16)
        dm = dmin.astype(np.float64)[..., None]
        mn = np.where(dm > 0, np.clip(np.rint(target / np.where(dm > 0, dm, 1.0)), 0, 15), 0).astype(np.int32)
        b[..., :16] = (sc | (mn << 4)).astype(np.uint8)
    else:
        sc, _ = _k4_unpack(b[..., 4:16])
        qmean = 7.5 if type_id == Q4_K else 15.5
        target = qmean * d[..., None] * sc
        dmin = (target.max(axis=-1) / 63.0).astype(np.float16)
        dm = dmin.astype(np.float64)[..., None]
        mn = np.where(dm > 0, np.clip(np.rint(target / np.where(dm > 0, dm, 1.0)), 0, 63), 0).astype(np.int32)
        b[..., 4:16] = _k4_pack(sc, mn)
    b[..., m_off:m_off + 2] = dmin[..., None].view(np.uint8)
    return b.reshape(N, -1)


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
