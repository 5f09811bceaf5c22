"""Known-answer blocks of the reference's own tests, restated as data.

Each builder returns the same bytes and expected values as the cited test in
swllm.cpp's tests/test_gguf.cpp.  Used against the oracle (CPU) and against
the CUDA library (GPU tests).
"""
from __future__ import annotations

import struct

import numpy as np

Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 2, 8, 10, 11, 12, 13, 14

# ggml_type_size / ggml_block_size, tests/test_gguf.cpp:168-183, 1474-1495
TYPE_SIZES = {Q4_0: 18, Q8_0: 34, Q2_K: 84, Q3_K: 110, Q4_K: 144, Q5_K: 176, Q6_K: 210}
BLOCK_SIZES = {Q4_0: 32, Q8_0: 32, Q2_K: 256, Q3_K: 256, Q4_K: 256, Q5_K: 256, Q6_K: 256}

# fp16 conversions, tests/test_gguf.cpp:248-267
FP16_CASES = [(0x0000, 0.0), (0x3C00, 1.0), (0xBC00, -1.0), (0x3800, 0.5), (0x4000, 2.0)]

ONE = 0x3C00
TWO = 0x4000


def _h(v: int) -> bytes:
    return struct.pack("<H", v)


def q8_0_2x32() -> dict:
    """tests/test_gguf.cpp:370-411: rows scale 1.0 / 2.0, values 1..32, x = 1."""
    rows = []
    for d in (ONE, TWO):
        rows.append(_h(d) + bytes(range(1, 33)))
    w = np.frombuffer(b"".join(rows), dtype=np.uint8).copy()
    return dict(type=Q8_0, blocks=w, N=2, K=32, x=np.ones(32, np.float32),
                expect=np.array([528.0, 1056.0], np.float32), tol=0.5)


def q4_0_2x32() -> dict:
    """tests/test_gguf.cpp:413-474: row 0 nibbles 0x88 (all 0), row 1 0x79
    (+1 for x[0..15], -1 for x[16..31]); x = 1 and x alternating +-1."""
    w = np.frombuffer(_h(ONE) + bytes([0x88] * 16) + _h(ONE) + bytes([0x79] * 16),
                      dtype=np.uint8).copy()
    x_alt = np.array([1.0 if j % 2 == 0 else -1.0 for j in range(32)], np.float32)
    return dict(type=Q4_0, blocks=w, N=2, K=32, x=np.ones(32, np.float32),
                expect=np.array([0.0, 0.0], np.float32), tol=1e-4, x_alt=x_alt)


def q6_k_block() -> np.ndarray:
    """tests/test_gguf.cpp:1500-1528: d = 1, scales = 1, ql = qh = 0 -> -32."""
    b = bytearray(210)
    for i in range(16):
        b[192 + i] = 1
    b[208:210] = _h(ONE)
    return np.frombuffer(bytes(b), dtype=np.uint8).copy()


def q4_k_block() -> np.ndarray:
    """tests/test_gguf.cpp:1534-1565: d = 1, dmin = 0, scales[0..3] = 1,
    qs = 0x88 -> first 128 outputs 8.0."""
    b = bytearray(144)
    b[0:2] = _h(ONE)
    b[2:4] = _h(0)
    b[4:8] = bytes([1, 1, 1, 1])
    for i in range(16, 144):
        b[i] = 0x88
    return np.frombuffer(bytes(b), dtype=np.uint8).copy()


def q2_k_block() -> np.ndarray:
    """tests/test_gguf.cpp:1568-1599: sc = 1, m = 0, qs = 0 -> all 0."""
    b = bytearray(84)
    for i in range(16):
        b[i] = 0x01
    b[80:82] = _h(ONE)
    b[82:84] = _h(0)
    return np.frombuffer(bytes(b), dtype=np.uint8).copy()


def q5_k_block() -> np.ndarray:
    """tests/test_gguf.cpp:1657-1687: d = 1, dmin = 0, scales[0..3] = 1,
    qh = 0, qs = 0x55 -> first 128 outputs 5.0."""
    b = bytearray(176)
    b[0:2] = _h(ONE)
    b[2:4] = _h(0)
    b[4:8] = bytes([1, 1, 1, 1])
    for i in range(48, 176):
        b[i] = 0x55
    return np.frombuffer(bytes(b), dtype=np.uint8).copy()


def dequant_kats() -> list[dict]:
    """(type, block, check) where check is (slice, expected value)."""
    return [
        dict(name="q6_k", type=Q6_K, blocks=q6_k_block(), n=256, sl=slice(0, 256), value=-32.0, tol=1e-4),
        dict(name="q4_k", type=Q4_K, blocks=q4_k_block(), n=256, sl=slice(0, 128), value=8.0, tol=1e-4),
        dict(name="q2_k", type=Q2_K, blocks=q2_k_block(), n=256, sl=slice(0, 256), value=0.0, tol=1e-5),
        dict(name="q5_k", type=Q5_K, blocks=q5_k_block(), n=256, sl=slice(0, 128), value=5.0, tol=1e-4),
    ]


def fused_kats() -> list[dict]:
    """Fused GEMV known answers, x = 1:
    Q6_K 2x256 -> -8192 (tests/test_gguf.cpp:1690-1729);
    Q4_K / Q5_K 2x256 vs dequantize-then-GEMV (:1732-1810)."""
    out = []
    out.append(dict(name="q6_k", type=Q6_K, blocks=np.concatenate([q6_k_block()] * 2), N=2, K=256,
                    expect=np.array([-8192.0, -8192.0], np.float32), tol=1e-1))
    out.append(dict(name="q4_k", type=Q4_K, blocks=np.concatenate([q4_k_block()] * 2), N=2, K=256,
                    expect=None, tol=1e-3))
    out.append(dict(name="q5_k", type=Q5_K, blocks=np.concatenate([q5_k_block()] * 2), N=2, K=256,
                    expect=None, tol=1e-3))
    return out
