"""The batched Q4_K / Q6_K GEMV (gemv_kqm.cu: 2..32 activation rows, each
weight read once for all rows) against the oracle restatements of
cpu_matmul_transposed_q4_k / _q6_k (src/tensor.h:769-856), row by row.

Per row, x is held relative to each super-block's largest element as two
fp16 parts (22 bits), every product with a quant value is exact and the sums
are fp32, so every output row is held to relative L2 1e-5 of the oracle's.
Shapes cover one to four blocks of 8 activation rows (odd M, zero padding
rows), K split over CTAs (partials summed by the last CTA of a row range)
and over the splits of one CTA (large N), Q6_K boxes that start below a block
(210-byte blocks), row counts that are not a multiple of 16 and CTAs with
fewer rows than a tile; the tuning options (table size, warps per tile)
change the split plan and the reduction, not the result."""
import numpy as np
import pytest

import swq
from conftest import rel_l2
from swq import synth

pytestmark = pytest.mark.gpu

F32 = np.float32
TOL = 1e-5


@pytest.fixture(autouse=True)
def _batched_form():
    old = [swq.get_option(o) for o in (swq.OPT_GEMV_BATCH_MAX_M, swq.OPT_GEMV_BATCH_TABLE_KB,
                                       swq.OPT_GEMV_BATCH_GROUP)]
    swq.set_option(swq.OPT_GEMV_BATCH_MAX_M, 32)
    yield
    for o, v in zip((swq.OPT_GEMV_BATCH_MAX_M, swq.OPT_GEMV_BATCH_TABLE_KB, swq.OPT_GEMV_BATCH_GROUP), old):
        swq.set_option(o, v)


def _check_rows(got, want, oracle_mod, t, blocks, X, N, K, tol=TOL):
    """Per activation row: rel-L2 against the oracle; for a few output rows
    (which can cancel far below their terms) each output against
    sum_k |w_k x_k| instead."""
    M = X.shape[0]
    got = np.asarray(got).reshape(M, N)
    want = np.asarray(want).reshape(M, N)
    if N >= 16:
        for m in range(M):
            assert rel_l2(got[m], want[m]) <= tol, (m, rel_l2(got[m], want[m]))
        return
    W = np.abs(oracle_mod.dequantize(t, blocks, N * K).reshape(N, K).astype(np.float64))
    scale = np.abs(np.asarray(X, np.float64)) @ W.T
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert (err <= 1e-6 * scale).all(), (err, scale)


def _run(torch, t, blocks, X, N, K, pad=0):
    M = X.shape[0]
    d_w = torch.from_numpy(np.ascontiguousarray(blocks).reshape(-1)).cuda()
    d_x = torch.from_numpy(np.ascontiguousarray(X, dtype=F32)).cuda()
    d_y = torch.full((M * N + pad,), float("nan"), dtype=torch.float32, device="cuda")
    swq.gemm(t, d_w, d_x, d_y, M, N, K)
    swq.check()
    return d_y.cpu().numpy()


SHAPES = [(300, 2048), (4096, 4096), (1024, 14336), (5000, 4096), (17, 2048), (16, 2048), (148 * 16 + 5, 4096)]


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("M", [2, 3, 5, 8, 9, 16, 17, 32])
@pytest.mark.parametrize("N,K", SHAPES)
def test_kqm_shapes(cuda, oracle_mod, fmt, M, N, K):
    t = synth.IDS[fmt]
    blocks = synth.random_blocks(t, N, K, seed=N + 3 * K + M)
    X = synth.random_activations(M, K, seed=K + M)
    got = _run(cuda, t, blocks, X, N, K, pad=64)
    assert np.isnan(got[M * N:]).all()  # nothing written past the M rows
    want = oracle_mod.gemm(t, blocks, X, M, N, K)
    _check_rows(got[:M * N], want, oracle_mod, t, blocks, X, N, K)


@pytest.mark.parametrize("fmt,M,N,K", [("Q4_K", 32, 20000, 4096), ("Q6_K", 16, 40000, 4096),
                                       ("Q4_K", 16, 2048, 28672), ("Q6_K", 4, 1000, 16384),
                                       ("Q4_K", 12, 9000, 4096)])
def test_kqm_large(cuda, oracle_mod, fmt, M, N, K):
    """Partials too large for L2 (one CTA runs every split of its rows, adding
    into Y in split order), and long rows split over many CTAs; at 9..16 rows
    the automatic plan takes the 144 KB table on all but the first shape."""
    t = synth.IDS[fmt]
    blocks = synth.random_blocks(t, N, K, seed=N + K)
    X = synth.random_activations(M, K, seed=M * 7)
    got = _run(cuda, t, blocks, X, N, K)
    want = oracle_mod.gemm(t, blocks, X, M, N, K)
    _check_rows(got, want, oracle_mod, t, blocks, X, N, K)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("table_kb,group", [(0, 0), (72, 1), (36, 0), (36, 2), (18, 1), (144, 4), (9, 0)])
@pytest.mark.parametrize("M,N,K", [(8, 3000, 4096), (16, 1000, 14336), (32, 700, 8192), (2, 24000, 2048)])
def test_kqm_tuning_plans(cuda, oracle_mod, fmt, table_kb, group, M, N, K):
    """Every table size and tile group gives the oracle's rows, also where a
    CTA's tiles go round the weight ring several times (24000 rows: the plan
    then keeps a tile's stages per group in the ring)."""
    t = synth.IDS[fmt]
    swq.set_option(swq.OPT_GEMV_BATCH_TABLE_KB, table_kb)
    swq.set_option(swq.OPT_GEMV_BATCH_GROUP, group)
    blocks = synth.random_blocks(t, N, K, seed=N + M + table_kb)
    X = synth.random_activations(M, K, seed=K + group)
    got = _run(cuda, t, blocks, X, N, K)
    _check_rows(got, oracle_mod.gemm(t, blocks, X, M, N, K), oracle_mod, t, blocks, X, N, K)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_kqm_matches_single_row_form(cuda, oracle_mod, fmt):
    """Each row agrees with the single-row integer kernel's result to 2e-6."""
    torch = cuda
    t = synth.IDS[fmt]
    M, N, K = 6, 4096, 4096
    blocks = synth.random_blocks(t, N, K, seed=41)
    X = synth.random_activations(M, K, seed=42)
    got = _run(torch, t, blocks, X, N, K).reshape(M, N)
    d_w = torch.from_numpy(blocks.reshape(-1)).cuda()
    for m in range(M):
        y = torch.empty(N, dtype=torch.float32, device="cuda")
        swq.gemv(t, d_w, torch.from_numpy(np.ascontiguousarray(X[m])).cuda(), y, N, K)
        swq.check()
        assert rel_l2(got[m], y.cpu().numpy()) <= 2e-6


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_kqm_deterministic_pool_and_workspace(cuda, fmt):
    """Repeated calls, and the pool and caller-workspace forms, give the same bits."""
    torch = cuda
    t = synth.IDS[fmt]
    M, N, K = 16, 4096, 14336
    blocks = synth.random_blocks(t, N, K, seed=43)
    X = synth.random_activations(M, K, seed=44)
    a = _run(torch, t, blocks, X, N, K)
    b = _run(torch, t, blocks, X, N, K)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    need = swq.gemm_workspace_bytes(t, M, N, K)
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    y = torch.full((M, N), float("nan"), device="cuda")
    swq.gemm_act_ws(t, torch.from_numpy(blocks.reshape(-1)).cuda(), torch.from_numpy(X).cuda(), y, M, N, K, ws, need)
    swq.check()
    assert np.array_equal(y.cpu().numpy().reshape(-1).view(np.uint32), a.view(np.uint32))
    with pytest.raises(swq.SwqError):  # a workspace one byte short
        swq.gemm_act_ws(t, torch.from_numpy(blocks.reshape(-1)).cuda(), torch.from_numpy(X).cuda(), y, M, N, K,
                        ws, need - 1)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_kqm_rows_independent_dynamic_range(cuda, oracle_mod, fmt):
    """Rows of very different magnitude, a zero row, a super-block of
    subnormals and a non-finite value in one row: every row gets its own
    scales, and only the row holding inf turns non-finite."""
    t = synth.IDS[fmt]
    M, N, K = 8, 512, 4096
    blocks = synth.random_blocks(t, N, K, seed=45)
    rng = np.random.default_rng(46)
    X = (rng.standard_normal((M, K)) * 10.0 ** rng.uniform(-6, 6, (M, K))).astype(F32)
    X[1] *= F32(1e-20)
    X[2] = 0.0
    X[3, 1024:1280] = F32(1e-40)
    X[5, 700] = np.inf
    got = _run(cuda, t, blocks, X, N, K).reshape(M, N)
    want = oracle_mod.gemm(t, blocks, X, M, N, K).reshape(M, N)
    for m in range(M):
        if m == 5:
            assert not np.isfinite(got[m]).any()
        elif m == 2:
            assert (got[m] == 0).all()
        else:
            assert rel_l2(got[m], want[m]) <= TOL, m


def _rms_ref(x, w, eps):
    ss = (x.astype(np.float64) ** 2).sum(axis=1, keepdims=True)
    return (x / np.sqrt(ss / x.shape[1] + eps) * w).astype(F32)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("M,N,K", [(5, 640, 2048), (16, 4096, 4096), (32, 1024, 8192)])
@pytest.mark.parametrize("residual", [False, True])
def test_kqm_rmsnorm_prologue(cuda, oracle_mod, fmt, M, N, K, residual):
    torch = cuda
    t = synth.IDS[fmt]
    rng = np.random.default_rng(N + M + residual)
    blocks = synth.random_blocks(t, N, K, seed=47)
    X = (rng.standard_normal((M, K)) * 3).astype(F32)
    R = rng.standard_normal((M, K)).astype(F32) if residual else None
    w = (1 + 0.1 * rng.standard_normal(K)).astype(F32)
    xs = X + R if residual else X
    want = oracle_mod.gemm(t, blocks, _rms_ref(xs, w, 1e-5), M, N, K)
    y = torch.full((M, N), float("nan"), device="cuda")
    so = torch.full((M, K), float("nan"), device="cuda")
    swq.gemm_act(t, torch.from_numpy(blocks.reshape(-1)).cuda(), torch.from_numpy(X).cuda(), y, M, N, K,
                 kind=swq.ACT_RMSNORM, residual=torch.from_numpy(R).cuda() if residual else None,
                 norm_w=torch.from_numpy(w).cuda(), eps=1e-5, sum_out=so)
    swq.check()
    _check_rows(y.cpu().numpy(), want, oracle_mod, t, blocks, X, N, K)
    assert np.array_equal(so.cpu().numpy(), xs)


@pytest.mark.parametrize("fmt,M,N,K", [("Q4_K", 8, 4096, 4096), ("Q6_K", 16, 4096, 14336), ("Q6_K", 3, 512, 2048)])
def test_kqm_swiglu_prologue(cuda, oracle_mod, fmt, M, N, K):
    torch = cuda
    t = synth.IDS[fmt]
    ld = 2 * K + 64
    rng = np.random.default_rng(K + M)
    blocks = synth.random_blocks(t, N, K, seed=48)
    GU = (rng.standard_normal((M, ld)) * 2).astype(F32)
    g, u = GU[:, :K].astype(np.float64), GU[:, K:2 * K].astype(np.float64)
    h = (g / (1 + np.exp(-g)) * u).astype(F32)
    want = oracle_mod.gemm(t, blocks, h, M, N, K)
    y = torch.full((M, N), float("nan"), device="cuda")
    swq.gemm_act(t, torch.from_numpy(blocks.reshape(-1)).cuda(), torch.from_numpy(GU).cuda(), y, M, N, K,
                 kind=swq.ACT_SWIGLU, ld=ld)
    swq.check()
    _check_rows(y.cpu().numpy(), want, oracle_mod, t, blocks, h, N, K)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_kqm_misaligned_activations(cuda, oracle_mod, fmt):
    """X at a 4-byte (not 16-byte) offset: scalar activation loads."""
    torch = cuda
    t = synth.IDS[fmt]
    M, N, K = 4, 333, 4096
    blocks = synth.random_blocks(t, N, K, seed=49)
    X = synth.random_activations(M, K, seed=50)
    buf = torch.zeros(M * K + 8, dtype=torch.float32, device="cuda")
    buf[1:M * K + 1] = torch.from_numpy(X.reshape(-1)).cuda()
    y = torch.full((M * N,), float("nan"), dtype=torch.float32, device="cuda")
    swq.gemm(t, torch.from_numpy(blocks.reshape(-1)).cuda(), buf.data_ptr() + 4, y, M, N, K)
    swq.check()
    _check_rows(y.cpu().numpy(), oracle_mod.gemm(t, blocks, X, M, N, K), oracle_mod, t, blocks, X, N, K)


def test_kqm_option_off_uses_other_paths(cuda, oracle_mod):
    """SWQ_OPT_GEMV_BATCH_MAX_M below M: the tensor-core GEMM (fp16 operands,
    1e-3) serves the call instead."""
    t = swq.Q4_K
    M, N, K = 16, 1024, 4096
    blocks = synth.random_blocks(t, N, K, seed=51)
    X = synth.random_activations(M, K, seed=52)
    want = np.asarray(oracle_mod.gemm(t, blocks, X, M, N, K)).reshape(M, N)
    swq.set_option(swq.OPT_GEMV_BATCH_MAX_M, 8)
    got = _run(cuda, t, blocks, X, N, K).reshape(M, N)
    assert rel_l2(got, want) <= 1e-3
    assert rel_l2(got, want) > TOL  # fp16 operands: not the batched form
