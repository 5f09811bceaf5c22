"""Tensor-core (tcgen05) dequant-GEMM against the oracle.

The reference has no batched quantized path: its prefill is one
Compute::matmul_transposed_q per token (src/main.cpp:284-287), so the oracle
for M rows is M such calls.  Tolerance: relative L2 <= 1e-3 (REL_L2_TOL); the
kernel rounds dequantized weights and activations to fp16 before an
fp32-accumulated product (expected ~3e-4).
"""
import numpy as np
import pytest

import swq
from conftest import REL_L2_TOL, rel_l2
from swq import synth

pytestmark = pytest.mark.gpu

FORMATS = ["Q4_0", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]


def _gemm(torch, t, blocks, X, N, K):
    M = X.shape[0]
    d_w = torch.from_numpy(np.ascontiguousarray(blocks).reshape(-1)).cuda()
    d_x = torch.from_numpy(np.ascontiguousarray(X, dtype=np.float32)).cuda()
    d_y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    swq.gemm(t, d_w, d_x, d_y, M, N, K)
    swq.check()
    return d_y.cpu().numpy()


@pytest.fixture(autouse=True)
def _tensor_core_on():
    """Every M above the GEMV limit takes the tensor-core path in these tests."""
    swq.set_option(swq.OPT_TENSOR_CORE_GEMM, 1)
    swq.set_option(swq.OPT_TENSOR_CORE_MIN_M, 9)
    yield
    swq.set_option(swq.OPT_TENSOR_CORE_GEMM, 1)
    swq.set_option(swq.OPT_TENSOR_CORE_MIN_M, 5)


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("M", [9, 64, 100, 130, 256])
def test_formats(cuda, oracle_mod, fmt, M):
    t = synth.IDS[fmt]
    qk, _ = synth.block_geometry(t)
    N, K = 384, 2048 if qk == 256 else 1024
    blocks = synth.random_blocks(t, N, K, seed=2000 + t)
    X = synth.random_activations(M, K, seed=2001 + M)
    got = _gemm(cuda, t, blocks, X, N, K)
    want = oracle_mod.gemm(t, blocks, X, M, N, K)
    err = rel_l2(got, want)
    assert err <= REL_L2_TOL, err
    assert np.all(np.isfinite(got))


@pytest.mark.parametrize("order", ["reference_cpu", "format"])
@pytest.mark.parametrize("M", [9, 130])
def test_q2k_orders(cuda, oracle_mod, order, M):
    """Q2_K on the tensor cores in both activation orders: the reference's
    fused CPU routine (default; the fp16 copy of X repeats the first 32
    elements of each 128-element half for all four planes) and
    dequantize_q2_k's order (SWQ_OPT_Q2K_REFERENCE_CPU_ORDER = 0)."""
    t = synth.IDS["Q2_K"]
    N, K = 384, 2048
    blocks = synth.random_blocks(t, N, K, seed=2050)
    X = synth.random_activations(M, K, seed=2051)
    fmt_order = order == "format"
    swq.set_option(swq.OPT_Q2K_REFERENCE_CPU_ORDER, 0 if fmt_order else 1)
    try:
        got = _gemm(cuda, t, blocks, X, N, K)
    finally:
        swq.set_option(swq.OPT_Q2K_REFERENCE_CPU_ORDER, 1)
    want = oracle_mod.gemm(t, blocks, X, M, N, K, format_order=fmt_order)
    other = oracle_mod.gemm(t, blocks, X, M, N, K, format_order=not fmt_order)
    assert rel_l2(got, want) <= REL_L2_TOL
    assert rel_l2(got, other) > 0.1  # the two orders are far apart


@pytest.mark.parametrize("fmt,N,K,M", [("Q4_K", 200, 512, 70), ("Q4_0", 129, 96, 33), ("Q8_0", 257, 160, 300),
                                        ("Q6_K", 130, 768, 17), ("Q5_K", 1000, 1280, 511)])
def test_ragged_tiles(cuda, oracle_mod, fmt, N, K, M):
    """N not a multiple of 128, M not a multiple of the token tile, K with an
    odd number of 32-element blocks (a half-filled last K step)."""
    t = synth.IDS[fmt]
    blocks = synth.random_blocks(t, N, K, seed=2100 + N)
    X = synth.random_activations(M, K, seed=2101)
    got = _gemm(cuda, t, blocks, X, N, K)
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, M, N, K)) <= REL_L2_TOL


@pytest.mark.parametrize("fmt,M", [("Q4_K", 512), ("Q6_K", 64), ("Q8_0", 64), ("Q4_0", 64), ("Q2_K", 64),
                                    ("Q3_K", 64), ("Q5_K", 64)])
def test_llama_ffn_shape(cuda, oracle_mod, fmt, M):
    """N=14336, K=4096 (Llama-3-8B FFN up-projection), prefill-sized M."""
    t = synth.IDS[fmt]
    N, K = 14336, 4096
    blocks = synth.random_blocks(t, N, K, seed=2200 + t)
    X = synth.random_activations(M, K, seed=2201)
    got = _gemm(cuda, t, blocks, X, N, K)
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, M, N, K)) <= REL_L2_TOL


@pytest.mark.parametrize("fmt,K,off", [("Q4_K", 1024, 8), ("Q4_K", 1024, 2), ("Q5_K", 2048, 4), ("Q6_K", 2048, 2),
                                        ("Q2_K", 768, 0), ("Q3_K", 1280, 0), ("Q8_0", 1024, 6), ("Q4_0", 1056, 2)])
def test_row_copies(cuda, oracle_mod, fmt, K, off):
    """Rows not 16-byte aligned (W offset from its allocation, or a row size
    that is not a multiple of 16): the W stages arrive as one copy per row and
    each row's blocks start part way into their shared-memory row."""
    torch = cuda
    t = synth.IDS[fmt]
    N, M = 200, 40
    blocks = synth.random_blocks(t, N, K, seed=2300 + off)
    X = synth.random_activations(M, K, seed=2301)
    flat = blocks.reshape(-1)
    d_w = torch.zeros(flat.size + 64, dtype=torch.uint8, device="cuda")
    d_w[off:off + flat.size] = torch.from_numpy(flat).cuda()
    d_x = torch.from_numpy(X).cuda()
    d_y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    swq.gemm(t, d_w.data_ptr() + off, d_x, d_y, M, N, K)
    swq.check()
    assert rel_l2(d_y.cpu().numpy(), oracle_mod.gemm(t, blocks, X, M, N, K)) <= REL_L2_TOL


def test_gemv_groups_when_disabled(cuda, oracle_mod):
    """SWQ_OPT_TENSOR_CORE_GEMM = 0: groups of rows through the GEMV kernel."""
    t = synth.Q4_K
    N, K, M = 256, 1024, 40
    blocks = synth.random_blocks(t, N, K, seed=2350)
    X = synth.random_activations(M, K, seed=2351)
    swq.set_option(swq.OPT_TENSOR_CORE_GEMM, 0)
    got = _gemm(cuda, t, blocks, X, N, K)
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, M, N, K)) <= REL_L2_TOL


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K", "Q8_0"])
def test_activations_beyond_fp16_range(cuda, oracle_mod, fmt):
    """Rows whose magnitudes exceed fp16's 65504 (a SwiGLU output of large
    gate/up values) next to ordinary, tiny and all-zero rows: each row is
    scaled by a power of two before the fp16 conversion, so every row keeps
    the relative accuracy of an ordinary one and nothing overflows."""
    t = synth.IDS[fmt]
    N, K, M = 256, 1024, 24
    blocks = synth.random_blocks(t, N, K, seed=2450 + t)
    X = synth.random_activations(M, K, seed=2451)
    X[1] *= 3.0e5
    X[2] *= 1.0e9
    X[3, 17] = 2.0e7
    X[4] *= 1.0e-6
    X[5] = 0.0
    X[6] *= 6.0e4
    got = _gemm(cuda, t, blocks, X, N, K)
    want = oracle_mod.gemm(t, blocks, X, M, N, K)
    assert np.all(np.isfinite(got))
    assert np.all(got[5] == 0.0)
    for r in range(M):
        if r == 5:
            continue
        assert rel_l2(got[r], want[r]) <= REL_L2_TOL, (r, rel_l2(got[r], want[r]))


@pytest.mark.parametrize("fmt,N,K,M", [("Q4_K", 4096, 4096, 16), ("Q6_K", 4096, 14336, 16), ("Q6_K", 1024, 4096, 9),
                                        ("Q4_K", 5120, 4096, 32), ("Q5_K", 640, 1280, 20), ("Q4_0", 300, 2336, 12),
                                        ("Q8_0", 256, 544, 64), ("Q2_K", 4096, 8192, 64), ("Q3_K", 1024, 3072, 100)])
def test_split_k(cuda, oracle_mod, fmt, N, K, M):
    """Output tiles fewer than half the SMs: K is split into parts whose
    partial tiles the last part sums (in split order) -- decode-batch shapes,
    an odd number of W stages, a Q4_0 K ending half way through a step, two
    token tiles."""
    t = synth.IDS[fmt]
    blocks = synth.random_blocks(t, N, K, seed=2500 + N + M)
    X = synth.random_activations(M, K, seed=2501)
    got = _gemm(cuda, t, blocks, X, N, K)
    assert np.all(np.isfinite(got))
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, M, N, K)) <= REL_L2_TOL


def test_split_k_deterministic(cuda):
    torch = cuda
    t = synth.Q6_K
    N, K, M = 4096, 14336, 16
    d_w = torch.from_numpy(synth.random_blocks(t, N, K, seed=2600).reshape(-1)).cuda()
    d_x = torch.from_numpy(synth.random_activations(M, K, seed=2601)).cuda()
    ys = [torch.empty((M, N), dtype=torch.float32, device="cuda") for _ in range(3)]
    for y in ys:
        swq.gemm(t, d_w, d_x, y, M, N, K)
    swq.check()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[1], ys[2])


def test_deterministic(cuda):
    torch = cuda
    t = synth.Q4_K
    N, K, M = 1024, 2048, 256
    d_w = torch.from_numpy(synth.random_blocks(t, N, K, seed=2400).reshape(-1)).cuda()
    d_x = torch.from_numpy(synth.random_activations(M, K, seed=2401)).cuda()
    ys = [torch.empty((M, N), dtype=torch.float32, device="cuda") for _ in range(3)]
    for y in ys:
        swq.gemm(t, d_w, d_x, y, M, N, K)
    swq.check()
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[1], ys[2])
