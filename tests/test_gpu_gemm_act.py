"""swq_gemm_act: the GEMM/GEMV with the activation prologue fused (RMSNorm
with the residual add, SwiGLU) against the oracle GEMM of the transformed
activations computed in numpy the reference's way (src/tensor.h:1028-1064).
GEMV (M <= 4) and tensor-core (M >= 5) paths, with and without the
allocation-free flag.  Tolerance: relative L2 1e-3 as for swq_gemm; the
residual sum is exact (one fp32 add)."""
import numpy as np
import pytest

import swq
from conftest import REL_L2_TOL, rel_l2
from swq import synth

pytestmark = pytest.mark.gpu

F32 = np.float32


def _rms_ref(x, w, eps):
    ss = (x.astype(np.float64) ** 2).sum(axis=1, keepdims=True)
    return (x / np.sqrt(ss / x.shape[1] + eps) * w).astype(F32)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K", "Q8_0"])
@pytest.mark.parametrize("M", [1, 3, 9, 40])
@pytest.mark.parametrize("residual", [False, True])
def test_rmsnorm_prologue(cuda, oracle_mod, fmt, M, residual):
    torch = cuda
    t = synth.IDS[fmt]
    N, K = 640, 2048
    rng = np.random.default_rng(M * 10 + residual)
    blocks = synth.random_blocks(t, N, K, seed=7000 + t)
    X = rng.standard_normal((M, K)).astype(F32) * 3
    R = rng.standard_normal((M, K)).astype(F32) if residual else None
    w = (1 + 0.1 * rng.standard_normal(K)).astype(F32)
    xs = X + R if residual else X
    want = oracle_mod.gemm(t, blocks, _rms_ref(xs, w, 1e-5), M, N, K)
    d_w = torch.from_numpy(blocks.reshape(-1)).cuda()
    d_x = torch.from_numpy(X).cuda()
    d_r = torch.from_numpy(R).cuda() if residual else None
    d_nw = torch.from_numpy(w).cuda()
    for noalloc in (False, True):
        y = torch.full((M, N), float("nan"), device="cuda")
        so = torch.full((M, K), float("nan"), device="cuda")
        swq.gemm_act(t, d_w, d_x, y, M, N, K, kind=swq.ACT_RMSNORM, residual=d_r, norm_w=d_nw, eps=1e-5,
                     sum_out=so, noalloc=noalloc)
        swq.check()
        assert rel_l2(y.cpu().numpy(), want) <= REL_L2_TOL
        assert np.array_equal(so.cpu().numpy(), xs)


@pytest.mark.parametrize("fmt", ["Q6_K", "Q4_K"])
@pytest.mark.parametrize("M", [1, 2, 16])
def test_swiglu_prologue(cuda, oracle_mod, fmt, M):
    torch = cuda
    t = synth.IDS[fmt]
    N, K = 512, 1536
    ld = 2 * K + 64  # rows wider than gate + up
    rng = np.random.default_rng(M)
    blocks = synth.random_blocks(t, N, K, seed=7100 + t)
    GU = (rng.standard_normal((M, ld)) * 2).astype(F32)
    g, u = GU[:, :K].astype(np.float64), GU[:, K:2 * K].astype(np.float64)
    h = (g / (1 + np.exp(-g)) * u).astype(F32)
    want = oracle_mod.gemm(t, blocks, h, M, N, K)
    y = torch.full((M, N), float("nan"), device="cuda")
    swq.gemm_act(t, torch.from_numpy(blocks.reshape(-1)).cuda(), torch.from_numpy(GU).cuda(), y, M, N, K,
                 kind=swq.ACT_SWIGLU, ld=ld)
    swq.check()
    assert rel_l2(y.cpu().numpy(), want) <= REL_L2_TOL


def test_act_none_is_gemm(cuda):
    torch = cuda
    t, N, K, M = synth.Q4_K, 300, 1024, 2
    d_w = torch.from_numpy(synth.random_blocks(t, N, K, seed=7200).reshape(-1)).cuda()
    d_x = torch.from_numpy(synth.random_activations(M, K, seed=7201)).cuda()
    y1, y2 = torch.empty((M, N), device="cuda"), torch.empty((M, N), device="cuda")
    swq.gemm(t, d_w, d_x, y1, M, N, K)
    swq.gemm_act(t, d_w, d_x, y2, M, N, K)
    swq.check()
    assert torch.equal(y1, y2)


def test_bad_prologue_arguments(cuda):
    torch = cuda
    w = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    x = torch.zeros((1, 256), device="cuda")
    y = torch.zeros((1, 4), device="cuda")
    with pytest.raises(swq.SwqError):
        swq.gemm_act(swq.Q4_K, w, x, y, 1, 4, 256, kind=swq.ACT_RMSNORM)  # no norm weights
    with pytest.raises(swq.SwqError):
        swq.gemm_act(swq.Q4_K, w, x, y, 1, 4, 256, kind=7)
    with pytest.raises(swq.SwqError):
        swq.gemm_act(swq.Q4_K, w, x, y, 1, 4, 256, kind=swq.ACT_SWIGLU, ld=300)  # ld < 2K


@pytest.mark.parametrize("fmt,M,N,K", [("Q4_K", 40, 640, 2048), ("Q6_K", 300, 1000, 4096), ("Q4_K", 3, 512, 1024),
                                       ("Q5_K", 3, 512, 1024), ("Q6_K", 12, 1000, 2048)])
def test_caller_workspace_matches_pool(cuda, fmt, M, N, K):
    """swq_gemm_act_ws with a workspace of exactly swq_gemm_workspace_bytes:
    the same kernels and split plan as the pool form, so the same bits (the
    CUDA-core GEMV rows, M <= 4 of the other formats, need no workspace; the
    batched K-quant GEMV needs one for its activation table)."""
    torch = cuda
    t = synth.IDS[fmt]
    d_w = torch.from_numpy(synth.random_blocks(t, N, K, seed=7300 + M).reshape(-1)).cuda()
    d_x = torch.from_numpy(synth.random_activations(M, K, seed=7301)).cuda()
    need = swq.gemm_workspace_bytes(t, M, N, K)
    batched = fmt in ("Q4_K", "Q6_K") and 2 <= M <= swq.get_option(swq.OPT_GEMV_BATCH_MAX_M)
    assert (need == 0) == (not batched and M < swq.get_option(swq.OPT_TENSOR_CORE_MIN_M))
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    y1, y2 = torch.empty((M, N), device="cuda"), torch.full((M, N), float("nan"), device="cuda")
    swq.gemm(t, d_w, d_x, y1, M, N, K)
    for _ in range(2):  # the workspace's counters are reset by the call itself
        swq.gemm_act_ws(t, d_w, d_x, y2, M, N, K, ws if need else None, need)
        swq.check()
        assert torch.equal(y1, y2)
    if need:
        with pytest.raises(swq.SwqError, match="needs"):
            swq.gemm_act_ws(t, d_w, d_x, y2, M, N, K, ws, need - 1)
        with pytest.raises(swq.SwqError):
            swq.gemm_act_ws(t, d_w, d_x, y2, M, N, K, None, 0)
        big = torch.empty(need + 512, dtype=torch.uint8, device="cuda")
        with pytest.raises(swq.SwqError, match="aligned"):
            swq.gemm_act_ws(t, d_w, d_x, y2, M, N, K, big.data_ptr() + 16, need)
