"""The single-row Q4_K / Q6_K GEMV with integer tensor-core sub-block sums
(gemv_kq.cu, SWQ_OPT_GEMV_INT_MMA >= 2) against the oracle restatements of
cpu_matmul_transposed_q4_k / _q6_k (src/tensor.h:769-856).

Its only roundings are the 30-bit fixed-point activations (per 256-element
super-block), one conversion per super-block and the fp32 sum over
super-blocks, so it is held to relative L2 1e-5 (the oracle's own fp32
rounding is of that order), not the matmul tolerance of 1e-3.  Shapes cover
one to seven weight chunks per row (a short last chunk, chunks of 4 and 8
super-blocks), one to thirteen 16-row tiles per CTA, row counts that are not
a multiple of 16, CTAs with fewer rows than a tile, and Q6_K blocks at both
alignments (210-byte blocks: every other one starts 2 bytes past a word)."""
import numpy as np
import pytest

import swq
from conftest import rel_l2
from swq import synth

pytestmark = pytest.mark.gpu

F32 = np.float32
TOL = 1e-5


@pytest.fixture(autouse=True)
def _q4k_form():
    old = swq.get_option(swq.OPT_GEMV_INT_MMA)
    swq.set_option(swq.OPT_GEMV_INT_MMA, 2)
    yield
    swq.set_option(swq.OPT_GEMV_INT_MMA, old)


def _check(got, want, oracle_mod, t, blocks, x, N, K):
    """rel-L2 against the oracle; a matrix of a few rows can have an output
    that cancels to far below its terms (one row of Q6_K 1 x 2048 sums to
    1.16 from terms of order 100), so there each output's error is measured
    against sum_k |w_k x_k| instead (the bound of any fp32 evaluation)."""
    if N >= 16:
        assert rel_l2(got, want) <= TOL
        return
    W = oracle_mod.dequantize(t, blocks, N * K).reshape(N, K).astype(np.float64)
    scale = np.abs(W) @ np.abs(np.asarray(x, np.float64).reshape(K))
    err = np.abs(np.asarray(got, np.float64).reshape(N) - np.asarray(want, np.float64).reshape(N))
    assert (err <= 1e-6 * scale).all(), (err, scale)


def _gemv(torch, blocks, x, N, K, t=swq.Q4_K):
    d_w = torch.from_numpy(np.ascontiguousarray(blocks).reshape(-1)).cuda()
    d_x = torch.from_numpy(np.ascontiguousarray(x, dtype=F32).reshape(-1)).cuda()
    d_y = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
    swq.gemv(t, d_w, d_x, d_y, N, K)
    swq.check()
    return d_y.cpu().numpy()


@pytest.mark.parametrize("N,K", [(4096, 4096), (14336, 4096), (1024, 4096), (300, 4096), (37, 1024),
                                 (1, 512), (2048, 512), (512, 2048), (1000, 8192), (4000, 7680),
                                 (148 * 16 + 5, 4096), (148 * 208 + 3, 1024)])
def test_q4k_shapes(cuda, oracle_mod, N, K):
    blocks = synth.random_blocks(swq.Q4_K, N, K, seed=N + 7 * K)
    x = synth.random_activations(1, K, seed=K)
    got = _gemv(cuda, blocks, x, N, K)
    want = oracle_mod.gemm(swq.Q4_K, blocks, x, 1, N, K)
    _check(got, want, oracle_mod, swq.Q4_K, blocks, x, N, K)


@pytest.mark.parametrize("N,K", [(4096, 14336), (32000, 4096), (1024, 4096), (300, 2048), (37, 8192),
                                 (1, 2048), (8192, 4096), (2000, 16384), (148 * 16 + 5, 4096), (148 * 40 + 3, 6144)])
def test_q6k_shapes(cuda, oracle_mod, N, K):
    blocks = synth.random_blocks(swq.Q6_K, N, K, seed=N + 5 * K)
    x = synth.random_activations(1, K, seed=K + 1)
    got = _gemv(cuda, blocks, x, N, K, swq.Q6_K)
    want = oracle_mod.gemm(swq.Q6_K, blocks, x, 1, N, K)
    _check(got, want, oracle_mod, swq.Q6_K, blocks, x, N, K)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_kq_dynamic_range(cuda, oracle_mod, fmt):
    """Activations over twelve decades, a super-block of zeros and one of
    subnormals: each super-block gets its own fixed-point scale."""
    t = synth.IDS[fmt]
    N, K = 200, 4096
    blocks = synth.random_blocks(t, N, K, seed=31)
    rng = np.random.default_rng(32)
    x = (rng.standard_normal(K) * 10.0 ** rng.uniform(-6, 6, K)).astype(F32)
    x[256:512] = 0.0
    x[1024:1280] = F32(1e-40)
    got = _gemv(cuda, blocks, x, N, K, t)
    want = oracle_mod.gemm(t, blocks, x.reshape(1, K), 1, N, K)
    assert rel_l2(got, want) <= TOL


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_kq_nonfinite_activation_propagates(cuda, oracle_mod, fmt):
    t = synth.IDS[fmt]
    N, K = 64, 2048
    blocks = synth.random_blocks(t, N, K, seed=33)
    x = synth.random_activations(1, K, seed=34)
    x[0, 700] = np.inf
    got = _gemv(cuda, blocks, x, N, K, t)
    want = oracle_mod.gemm(t, blocks, x, 1, N, K)
    assert not np.isfinite(want).any()
    assert not np.isfinite(got).any()


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_kq_deterministic_and_matches_cuda_core_form(cuda, oracle_mod, fmt):
    """Repeated calls give the same bits; the CUDA-core fp32 form agrees to
    the fp32 tolerance."""
    t = synth.IDS[fmt]
    N, K = 4096, 4096
    blocks = synth.random_blocks(t, N, K, seed=35)
    x = synth.random_activations(1, K, seed=36)
    a = _gemv(cuda, blocks, x, N, K, t)
    b = _gemv(cuda, blocks, x, N, K, t)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    swq.set_option(swq.OPT_GEMV_INT_MMA, 0)
    c = _gemv(cuda, blocks, x, N, K, t)
    assert rel_l2(a, c) <= TOL


def _rms_ref(x, w, eps):
    ss = (x.astype(np.float64) ** 2).sum(axis=1, keepdims=True)
    return (x / np.sqrt(ss / x.shape[1] + eps) * w).astype(F32)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("N,K", [(640, 2048), (4096, 4096), (1024, 8192)])
@pytest.mark.parametrize("residual", [False, True])
def test_kq_rmsnorm_prologue(cuda, oracle_mod, fmt, N, K, residual):
    torch = cuda
    t = synth.IDS[fmt]
    rng = np.random.default_rng(N + residual)
    blocks = synth.random_blocks(t, N, K, seed=37)
    X = (rng.standard_normal((1, K)) * 3).astype(F32)
    R = rng.standard_normal((1, K)).astype(F32) if residual else None
    w = (1 + 0.1 * rng.standard_normal(K)).astype(F32)
    xs = X + R if residual else X
    want = oracle_mod.gemm(t, blocks, _rms_ref(xs, w, 1e-5), 1, N, K)
    y = torch.full((1, N), float("nan"), device="cuda")
    so = torch.full((1, K), float("nan"), device="cuda")
    swq.gemm_act(t, torch.from_numpy(blocks.reshape(-1)).cuda(), torch.from_numpy(X).cuda(), y, 1, N, K,
                 kind=swq.ACT_RMSNORM, residual=torch.from_numpy(R).cuda() if residual else None,
                 norm_w=torch.from_numpy(w).cuda(), eps=1e-5, sum_out=so)
    swq.check()
    assert rel_l2(y.cpu().numpy(), want) <= TOL
    assert np.array_equal(so.cpu().numpy(), xs)


@pytest.mark.parametrize("fmt,N,K", [("Q4_K", 512, 1024), ("Q4_K", 4096, 4096), ("Q6_K", 4096, 14336),
                                     ("Q6_K", 512, 2048)])
def test_kq_swiglu_prologue(cuda, oracle_mod, fmt, N, K):
    torch = cuda
    t = synth.IDS[fmt]
    ld = 2 * K + 64
    rng = np.random.default_rng(K)
    blocks = synth.random_blocks(t, N, K, seed=38)
    GU = (rng.standard_normal((1, ld)) * 2).astype(F32)
    g, u = GU[:, :K].astype(np.float64), GU[:, K:2 * K].astype(np.float64)
    h = (g / (1 + np.exp(-g)) * u).astype(F32)
    want = oracle_mod.gemm(t, blocks, h, 1, N, K)
    y = torch.full((1, N), float("nan"), device="cuda")
    swq.gemm_act(t, torch.from_numpy(blocks.reshape(-1)).cuda(), torch.from_numpy(GU).cuda(), y, 1, N, K,
                 kind=swq.ACT_SWIGLU, ld=ld)
    swq.check()
    assert rel_l2(y.cpu().numpy(), want) <= TOL


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_kq_misaligned_activations(cuda, oracle_mod, fmt):
    """x at a 4-byte (not 16-byte) offset: scalar activation loads."""
    torch = cuda
    t = synth.IDS[fmt]
    N, K = 333, 4096
    blocks = synth.random_blocks(t, N, K, seed=39)
    x = synth.random_activations(1, K, seed=40)
    buf = torch.zeros(K + 8, dtype=torch.float32, device="cuda")
    buf[1:K + 1] = torch.from_numpy(x.reshape(-1)).cuda()
    y = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
    swq.gemv(t, torch.from_numpy(blocks.reshape(-1)).cuda(), buf.data_ptr() + 4, y, N, K)
    swq.check()
    assert rel_l2(y.cpu().numpy(), oracle_mod.gemm(t, blocks, x, 1, N, K)) <= TOL
