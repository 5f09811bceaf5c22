"""Seeded synthetic blocks follow the benchmark value distributions."""
import numpy as np
import pytest

from swq import synth


@pytest.mark.parametrize("t", list(synth.LAYOUT))
def test_shapes_and_determinism(t):
    qk, bb = synth.block_geometry(t)
    a = synth.random_blocks(t, 5, 4 * qk, seed=3)
    b = synth.random_blocks(t, 5, 4 * qk, seed=3)
    assert a.shape == (5, 4 * bb) and a.dtype == np.uint8
    assert np.array_equal(a, b)
    assert synth.matrix_bytes(t, 5, 4 * qk) == a.size


def test_q4k_scale_distribution(oracle_mod):
    t = synth.Q4_K
    blocks = synth.random_blocks(t, 64, 4096, seed=0).reshape(-1, 144)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    dm = blocks[:, 2:4].copy().view(np.float16).astype(np.float32).ravel()
    assert np.all(d >= 0) and np.all(dm >= 0)
    # |N(0,1)| mean is sqrt(2/pi) ~ 0.798
    assert abs(d.mean() / 2e-3 - 0.798) < 0.02
    assert abs(dm.mean() / 1e-3 - 0.798) < 0.02
    lib = oracle_mod.oracle_lib()
    import ctypes
    sc = ctypes.c_uint8()
    m = ctypes.c_uint8()
    seen = set()
    for blk in blocks[:200]:
        s = np.ascontiguousarray(blk[4:16])
        for j in range(8):
            lib.oracle_get_scale_min_k4(j, s.ctypes.data, ctypes.byref(sc), ctypes.byref(m))
            assert 0 <= sc.value < 64 and 0 <= m.value < 64
            seen.add(sc.value)
    assert len(seen) == 64


def test_q8_0_values_in_range():
    blocks = synth.random_blocks(synth.Q8_0, 32, 1024, seed=1).reshape(-1, 34)
    q = blocks[:, 2:].view(np.int8)
    assert q.min() >= -127 and q.max() <= 127


def test_bad_k():
    with pytest.raises(ValueError):
        synth.random_blocks(synth.Q4_K, 2, 100)
