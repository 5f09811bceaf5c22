"""swq_dequant on the GPU: bit-exact with the reference dequantize()."""
import numpy as np
import pytest

import kat
import swq
from conftest import GOLDEN
from swq import synth

pytestmark = pytest.mark.gpu

FORMATS = ["Q4_0", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]


def _dequant_gpu(torch, t, blocks, n, offset=0, fill=np.nan):
    d_blocks = torch.from_numpy(np.ascontiguousarray(blocks).reshape(-1)).cuda()
    out = torch.full((n + offset,), float(fill), dtype=torch.float32, device="cuda")
    swq.dequant(t, d_blocks, out.data_ptr() + 4 * offset, n)
    swq.check()
    return out.cpu().numpy()[offset:]


@pytest.mark.parametrize("fmt", FORMATS)
def test_random_blocks_bit_exact(cuda, oracle_mod, fmt):
    t = synth.IDS[fmt]
    N, K = 67, 4096
    blocks = synth.random_blocks(t, N, K, seed=11 + t)
    got = _dequant_gpu(cuda, t, blocks, N * K)
    want = oracle_mod.dequantize(t, blocks, N * K)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("fmt", FORMATS)
def test_golden_bit_exact(cuda, golden, fmt):
    g = golden(fmt)
    t, N, K = int(g["type"]), int(g["N"]), int(g["K"])
    got = _dequant_gpu(cuda, t, g["blocks"], N * K)
    assert np.array_equal(got.view(np.uint32), g["dequant"].view(np.uint32))


def test_special_scales_bit_exact(cuda):
    g = dict(np.load(GOLDEN / "golden_special_scales.npz"))
    for name in ("Q4_K", "Q6_K", "Q8_0"):
        t = synth.IDS[name]
        qk, bb = synth.block_geometry(t)
        blocks = g[f"{name}_blocks"]
        n = blocks.size // bb * qk
        got = _dequant_gpu(cuda, t, blocks, n)
        want = g[f"{name}_dequant"]
        # NaN results: x86 SSE yields the 'real indefinite' 0xFFC00000 for an
        # invalid operation (Inf * 0) and propagates input NaN payloads; the GPU
        # yields its canonical NaN.  Every other value, Inf and signed zero
        # included, must match bit for bit, and NaN must appear at the same places.
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan), name
        assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32)), name
        assert np.isinf(want).any() and nan.any()


@pytest.mark.parametrize("case", kat.dequant_kats(), ids=lambda c: c["name"])
def test_known_answers(cuda, case):
    got = _dequant_gpu(cuda, case["type"], case["blocks"], case["n"])
    np.testing.assert_allclose(got[case["sl"]], case["value"], atol=case["tol"])


@pytest.mark.parametrize("fmt", ["Q4_0", "Q4_K", "Q6_K"])
def test_tail_and_unaligned_output(cuda, oracle_mod, fmt):
    t = synth.IDS[fmt]
    qk, _ = synth.block_geometry(t)
    blocks = synth.random_blocks(t, 1, 8 * qk, seed=5)
    n = 8 * qk - 7  # the reference writes n / QK whole blocks; the tail is untouched
    got = _dequant_gpu(cuda, t, blocks, n, offset=1, fill=-7.0)
    want = oracle_mod.dequantize(t, blocks, 8 * qk)
    full = (n // qk) * qk
    assert np.array_equal(got[:full].view(np.uint32), want[:full].view(np.uint32))
    assert np.all(got[full:] == -7.0)


def test_zero_elements_is_noop(cuda):
    swq.dequant(synth.Q4_K, 0, 0, 0)
    swq.check()
