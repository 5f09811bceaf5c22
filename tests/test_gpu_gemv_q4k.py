"""The single-row Q4_K GEMV with integer tensor-core sub-block sums
(gemv_q4k.cu, SWQ_OPT_GEMV_INT_MMA >= 2) against the oracle restatement of
cpu_matmul_transposed_q4_k (src/tensor.h:817-856).

Its only roundings are the 30-bit fixed-point activations (per 256-element
super-block), one conversion per super-block and the fp32 sum over
super-blocks, so it is held to relative L2 1e-5 (the oracle's own fp32
rounding is of that order), not the matmul tolerance of 1e-3.  Shapes cover
one, two and three weight chunks per row (a short last chunk), one to
thirteen 16-row tiles per CTA, row counts that are not a multiple of 16 and
CTAs with fewer rows than a tile."""
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


def _gemv(torch, blocks, x, N, K):
    d_w = torch.from_numpy(np.ascontiguousarray(blocks).reshape(-1)).cuda()
    d_x = torch.from_numpy(np.ascontiguousarray(x, dtype=F32).reshape(-1)).cuda()
    d_y = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
    swq.gemv(swq.Q4_K, d_w, d_x, d_y, N, K)
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
    assert rel_l2(got, want) <= TOL


def test_q4k_dynamic_range(cuda, oracle_mod):
    """Activations over twelve decades, a super-block of zeros and one of
    subnormals: each super-block gets its own fixed-point scale."""
    N, K = 200, 4096
    blocks = synth.random_blocks(swq.Q4_K, N, K, seed=31)
    rng = np.random.default_rng(32)
    x = (rng.standard_normal(K) * 10.0 ** rng.uniform(-6, 6, K)).astype(F32)
    x[256:512] = 0.0
    x[1024:1280] = F32(1e-40)
    got = _gemv(cuda, blocks, x, N, K)
    want = oracle_mod.gemm(swq.Q4_K, blocks, x.reshape(1, K), 1, N, K)
    assert rel_l2(got, want) <= TOL


def test_q4k_nonfinite_activation_propagates(cuda, oracle_mod):
    N, K = 64, 2048
    blocks = synth.random_blocks(swq.Q4_K, N, K, seed=33)
    x = synth.random_activations(1, K, seed=34)
    x[0, 700] = np.inf
    got = _gemv(cuda, blocks, x, N, K)
    want = oracle_mod.gemm(swq.Q4_K, blocks, x, 1, N, K)
    assert not np.isfinite(want).any()
    assert not np.isfinite(got).any()


def test_q4k_deterministic_and_matches_cuda_core_form(cuda, oracle_mod):
    """Repeated calls give the same bits; the CUDA-core fp32 form agrees to
    the fp32 tolerance."""
    N, K = 4096, 4096
    blocks = synth.random_blocks(swq.Q4_K, N, K, seed=35)
    x = synth.random_activations(1, K, seed=36)
    a = _gemv(cuda, blocks, x, N, K)
    b = _gemv(cuda, blocks, x, N, K)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    swq.set_option(swq.OPT_GEMV_INT_MMA, 0)
    c = _gemv(cuda, blocks, x, N, K)
    assert rel_l2(a, c) <= TOL


def _rms_ref(x, w, eps):
    ss = (x.astype(np.float64) ** 2).sum(axis=1, keepdims=True)
    return (x / np.sqrt(ss / x.shape[1] + eps) * w).astype(F32)


@pytest.mark.parametrize("N,K", [(640, 2048), (4096, 4096), (1024, 8192)])
@pytest.mark.parametrize("residual", [False, True])
def test_q4k_rmsnorm_prologue(cuda, oracle_mod, N, K, residual):
    torch = cuda
    rng = np.random.default_rng(N + residual)
    blocks = synth.random_blocks(swq.Q4_K, N, K, seed=37)
    X = (rng.standard_normal((1, K)) * 3).astype(F32)
    R = rng.standard_normal((1, K)).astype(F32) if residual else None
    w = (1 + 0.1 * rng.standard_normal(K)).astype(F32)
    xs = X + R if residual else X
    want = oracle_mod.gemm(swq.Q4_K, blocks, _rms_ref(xs, w, 1e-5), 1, N, K)
    y = torch.full((1, N), float("nan"), device="cuda")
    so = torch.full((1, K), float("nan"), device="cuda")
    swq.gemm_act(swq.Q4_K, torch.from_numpy(blocks.reshape(-1)).cuda(), torch.from_numpy(X).cuda(), y, 1, N, K,
                 kind=swq.ACT_RMSNORM, residual=torch.from_numpy(R).cuda() if residual else None,
                 norm_w=torch.from_numpy(w).cuda(), eps=1e-5, sum_out=so)
    swq.check()
    assert rel_l2(y.cpu().numpy(), want) <= TOL
    assert np.array_equal(so.cpu().numpy(), xs)


@pytest.mark.parametrize("N,K", [(512, 1536 - 512), (4096, 4096)])
def test_q4k_swiglu_prologue(cuda, oracle_mod, N, K):
    torch = cuda
    ld = 2 * K + 64
    rng = np.random.default_rng(K)
    blocks = synth.random_blocks(swq.Q4_K, N, K, seed=38)
    GU = (rng.standard_normal((1, ld)) * 2).astype(F32)
    g, u = GU[:, :K].astype(np.float64), GU[:, K:2 * K].astype(np.float64)
    h = (g / (1 + np.exp(-g)) * u).astype(F32)
    want = oracle_mod.gemm(swq.Q4_K, blocks, h, 1, N, K)
    y = torch.full((1, N), float("nan"), device="cuda")
    swq.gemm_act(swq.Q4_K, torch.from_numpy(blocks.reshape(-1)).cuda(), torch.from_numpy(GU).cuda(), y, 1, N, K,
                 kind=swq.ACT_SWIGLU, ld=ld)
    swq.check()
    assert rel_l2(y.cpu().numpy(), want) <= TOL


def test_q4k_misaligned_activations(cuda, oracle_mod):
    """x at a 4-byte (not 16-byte) offset: scalar activation loads."""
    torch = cuda
    N, K = 333, 4096
    blocks = synth.random_blocks(swq.Q4_K, N, K, seed=39)
    x = synth.random_activations(1, K, seed=40)
    buf = torch.zeros(K + 8, dtype=torch.float32, device="cuda")
    buf[1:K + 1] = torch.from_numpy(x.reshape(-1)).cuda()
    y = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
    swq.gemv(swq.Q4_K, torch.from_numpy(blocks.reshape(-1)).cuda(), buf.data_ptr() + 4, y, N, K)
    swq.check()
    assert rel_l2(y.cpu().numpy(), oracle_mod.gemm(swq.Q4_K, blocks, x, 1, N, K)) <= TOL
