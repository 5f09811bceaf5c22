"""Fused dequant-GEMV / small-M GEMM on the GPU against the oracle.

Tolerance: relative L2 <= 1e-3 against the reference's fp32 result on the same
seeded inputs (REL_L2_TOL).  Q2_K is compared in the activation order of
the reference's fused CPU routine (the default, what
Compute::matmul_transposed_q returns) and, with
SWQ_OPT_Q2K_REFERENCE_CPU_ORDER = 0, in the element order of dequantize_q2_k.
"""
import numpy as np
import pytest

import kat
import swq
from conftest import REL_L2_TOL, rel_l2
from swq import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gemv_kernel_for_every_m():
    """These tests cover the GEMV kernel: keep every M off the tensor-core path."""
    swq.set_option(swq.OPT_TENSOR_CORE_MIN_M, 1 << 20)
    yield
    swq.set_option(swq.OPT_TENSOR_CORE_MIN_M, 5)

FORMATS = ["Q4_0", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]


def _gemm_gpu(torch, t, blocks, X, N, K, w_offset=0):
    M = X.shape[0]
    flat = np.ascontiguousarray(blocks).reshape(-1)
    d_w = torch.zeros(flat.size + 64, dtype=torch.uint8, device="cuda")
    d_w[w_offset:w_offset + flat.size] = torch.from_numpy(flat).cuda()
    d_x = torch.from_numpy(np.ascontiguousarray(X, dtype=np.float32)).cuda()
    d_y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    swq.gemm(t, d_w.data_ptr() + w_offset, d_x, d_y, M, N, K)
    swq.check()
    return d_y.cpu().numpy()


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("M", [1, 2, 3, 8])
def test_small_shapes(cuda, oracle_mod, fmt, M):
    t = synth.IDS[fmt]
    qk, _ = synth.block_geometry(t)
    N, K = 301, 8 * qk if qk == 256 else 64 * qk
    blocks = synth.random_blocks(t, N, K, seed=100 + t)
    X = synth.random_activations(M, K, seed=200 + M)
    got = _gemm_gpu(cuda, t, blocks, X, N, K)
    want = oracle_mod.gemm(t, blocks, X, M, N, K)
    assert rel_l2(got, want) <= REL_L2_TOL


@pytest.mark.parametrize("fmt", FORMATS)
def test_llama_ffn_shape_m1(cuda, oracle_mod, fmt):
    """N=14336, K=4096 (Llama-3-8B FFN up-projection), one activation row."""
    t = synth.IDS[fmt]
    N, K = 14336, 4096
    blocks = synth.random_blocks(t, N, K, seed=300 + t)
    X = synth.random_activations(1, K, seed=301)
    got = _gemm_gpu(cuda, t, blocks, X, N, K)
    want = oracle_mod.gemm(t, blocks, X, 1, N, K)
    assert rel_l2(got, want) <= REL_L2_TOL
    assert np.all(np.isfinite(got))


def test_q4k_4096_square(cuda, oracle_mod):
    t = synth.Q4_K
    blocks = synth.random_blocks(t, 4096, 4096, seed=0)
    X = synth.random_activations(1, 4096, seed=1)
    got = _gemm_gpu(cuda, t, blocks, X, 4096, 4096)
    want = oracle_mod.gemm(t, blocks, X, 1, 4096, 4096)
    err = rel_l2(got, want)
    assert err <= REL_L2_TOL
    # the fixed-point activation path is far inside the tolerance
    assert err < 1e-4


@pytest.mark.parametrize("fmt,K", [("Q6_K", 28672), ("Q4_K", 28672), ("Q4_K", 8192), ("Q8_0", 14336)])
def test_long_rows(cuda, oracle_mod, fmt, K):
    t = synth.IDS[fmt]
    N = 96
    blocks = synth.random_blocks(t, N, K, seed=400 + t)
    X = synth.random_activations(2, K, seed=401)
    got = _gemm_gpu(cuda, t, blocks, X, N, K)
    want = oracle_mod.gemm(t, blocks, X, 2, N, K)
    assert rel_l2(got, want) <= REL_L2_TOL


@pytest.mark.parametrize("fmt", FORMATS)
def test_golden_vectors(cuda, golden, fmt):
    g = golden(fmt)
    t, N, K = int(g["type"]), int(g["N"]), int(g["K"])
    got = _gemm_gpu(cuda, t, g["blocks"], g["x"], N, K)
    assert rel_l2(got, g["gemv_ref"]) <= REL_L2_TOL


def test_q2k_format_order_option(cuda, golden):
    """SWQ_OPT_Q2K_REFERENCE_CPU_ORDER = 0: dequantize_q2_k's element order,
    the reference's dequantize followed by an fp32 GEMV."""
    g = golden("Q2_K")
    t, N, K = int(g["type"]), int(g["N"]), int(g["K"])
    swq.set_option(swq.OPT_Q2K_REFERENCE_CPU_ORDER, 0)
    try:
        got = _gemm_gpu(cuda, t, g["blocks"], g["x"], N, K)
    finally:
        swq.set_option(swq.OPT_Q2K_REFERENCE_CPU_ORDER, 1)
    assert rel_l2(got, g["gemv_dq"]) <= REL_L2_TOL


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K", "Q2_K", "Q8_0"])
def test_unaligned_weights_and_rows(cuda, oracle_mod, fmt):
    """Base not 16-byte aligned, and rows whose byte length is not a multiple
    of 16 (one Q6_K/Q8_0 block per row): the plain-load producer path."""
    t = synth.IDS[fmt]
    qk, _ = synth.block_geometry(t)
    for N, K, off in ((37, qk, 0), (37, 3 * qk, 2), (64, 16 * qk if qk == 32 else 4 * qk, 6)):
        blocks = synth.random_blocks(t, N, K, seed=500 + off)
        X = synth.random_activations(3, K, seed=501)
        got = _gemm_gpu(cuda, t, blocks, X, N, K, w_offset=off)
        want = oracle_mod.gemm(t, blocks, X, 3, N, K)
        assert rel_l2(got, want) <= REL_L2_TOL, (N, K, off)


@pytest.mark.parametrize("N", [1, 7, 148, 149, 300])
def test_row_counts_around_grid(cuda, oracle_mod, N):
    t = synth.Q4_K
    blocks = synth.random_blocks(t, N, 1024, seed=600 + N)
    X = synth.random_activations(1, 1024, seed=601)
    got = _gemm_gpu(cuda, t, blocks, X, N, 1024)
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, 1, N, 1024)) <= REL_L2_TOL


def test_without_early_prefetch(cuda, oracle_mod):
    t = synth.Q5_K
    blocks = synth.random_blocks(t, 512, 2048, seed=7)
    X = synth.random_activations(4, 2048, seed=8)
    swq.set_option(swq.OPT_EARLY_WEIGHT_PREFETCH, 0)
    try:
        got = _gemm_gpu(cuda, t, blocks, X, 512, 2048)
    finally:
        swq.set_option(swq.OPT_EARLY_WEIGHT_PREFETCH, 1)
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, 4, 512, 2048)) <= REL_L2_TOL


@pytest.mark.parametrize("M", [9, 16, 64])
def test_larger_m(cuda, oracle_mod, M):
    t = synth.Q4_K
    N, K = 384, 2048
    blocks = synth.random_blocks(t, N, K, seed=700 + M)
    X = synth.random_activations(M, K, seed=701)
    got = _gemm_gpu(cuda, t, blocks, X, N, K)
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, M, N, K)) <= REL_L2_TOL


def test_back_to_back_launches_deterministic(cuda):
    torch = cuda
    t = synth.Q4_K
    N, K = 4096, 4096
    blocks = synth.random_blocks(t, N, K, seed=9)
    d_w = torch.from_numpy(blocks.reshape(-1)).cuda()
    d_x = torch.from_numpy(synth.random_activations(1, K, seed=10)).cuda()
    ys = [torch.empty(N, dtype=torch.float32, device="cuda") for _ in range(6)]
    for y in ys:
        swq.gemv(t, d_w, d_x, y, N, K)
    swq.check()
    for y in ys[1:]:
        assert torch.equal(y, ys[0])


def test_fused_known_answers(cuda):
    c = kat.q8_0_2x32()
    got = _gemm_gpu(cuda, c["type"], c["blocks"], c["x"][None, :], 2, 32)[0]
    np.testing.assert_allclose(got, c["expect"], atol=c["tol"])
    c = kat.q4_0_2x32()
    for x in (c["x"], c["x_alt"]):
        got = _gemm_gpu(cuda, c["type"], c["blocks"], x[None, :], 2, 32)[0]
        np.testing.assert_allclose(got, [0.0, 0.0], atol=1e-4)
    for case in kat.fused_kats():
        x = np.ones((1, case["K"]), np.float32)
        got = _gemm_gpu(cuda, case["type"], case["blocks"], x, case["N"], case["K"])[0]
        import oracle
        want = oracle.gemv(case["type"], case["blocks"], x[0], case["N"], case["K"])
        np.testing.assert_allclose(got, want, rtol=1e-3, atol=case["tol"])


@pytest.mark.parametrize("fmt,M", [("Q4_K", 1), ("Q6_K", 1), ("Q4_K", 4), ("Q6_K", 12), ("Q4_K", 40), ("Q5_K", 1)])
def test_host_buffer_repeated_calls(cuda, oracle_mod, fmt, M):
    """The host-buffer context over many calls in a row: new activations each
    time and two weights in turn, a larger shape in between (the staging
    buffers grow), an eviction, then the same shapes again -- every result the
    oracle's, on each path (integer GEMV, batched GEMV, tensor-core GEMM,
    CUDA-core GEMV)."""
    t = synth.IDS[fmt]
    N, K = 700, 4096
    ws = [swq.QuantWeight(synth.random_blocks(t, N, K, seed=20 + i), t) for i in range(2)]
    tol = REL_L2_TOL if M < 17 else 1e-3
    with swq.Compute() as c:
        for rnd in range(2):
            for i in range(5):
                X = synth.random_activations(M, K, seed=100 * rnd + i)
                Y = np.zeros((M, N), np.float32)
                w = ws[i % 2]
                c.matmul_q_batched(Y, X, w, M, N, K)
                assert rel_l2(Y, oracle_mod.gemm(t, w.data, X, M, N, K)) <= tol, (rnd, i)
            big = swq.QuantWeight(synth.random_blocks(t, 2 * N, 2 * K, seed=30 + rnd), t)
            X = synth.random_activations(M + 1, 2 * K, seed=7 + rnd)
            Y = np.zeros((M + 1, 2 * N), np.float32)
            c.matmul_q_batched(Y, X, big, M + 1, 2 * N, 2 * K)
            assert rel_l2(Y, oracle_mod.gemm(t, big.data, X, M + 1, 2 * N, 2 * K)) <= tol
            c.evict(ws[0])


def test_host_buffer_compute_api(cuda, oracle_mod):
    """Compute.matmul_transposed_q with host arrays, the reference's calling
    convention (src/tensor.h:1212): weights uploaded once and kept resident."""
    t = synth.Q6_K
    N, K = 1024, 4096
    w = swq.QuantWeight(synth.random_blocks(t, N, K, seed=12), t)
    x = synth.random_activations(1, K, seed=13)[0]
    out = np.zeros(N, np.float32)
    with swq.Compute() as c:
        c.matmul_transposed_q(out, x, w, N, K)
        assert rel_l2(out, oracle_mod.gemv(t, w.data, x, N, K)) <= REL_L2_TOL
        resident = c.resident_bytes()
        assert resident == synth.matrix_bytes(t, N, K)
        x2 = synth.random_activations(1, K, seed=14)[0]
        c.matmul_transposed_q(out, x2, w, N, K)
        assert c.resident_bytes() == resident  # cache hit, no second upload
        assert rel_l2(out, oracle_mod.gemv(t, w.data, x2, N, K)) <= REL_L2_TOL
        X = synth.random_activations(5, K, seed=15)
        Y = np.zeros((5, N), np.float32)
        c.matmul_q_batched(Y, X, w, 5, N, K)
        assert rel_l2(Y, oracle_mod.gemm(t, w.data, X, 5, N, K)) <= REL_L2_TOL
        c.evict(w)
        assert c.resident_bytes() == 0
        dst = np.zeros(N * K, np.float32)
        c.dequantize(w.data, dst, N * K, t)
        want = oracle_mod.dequantize(t, w.data, N * K)
        assert np.array_equal(dst.view(np.uint32), want.view(np.uint32))


def test_module_dequantize_host(cuda, oracle_mod):
    t = synth.Q3_K
    blocks = synth.random_blocks(t, 4, 1024, seed=16)
    dst = np.zeros(4096, np.float32)
    swq.dequantize(blocks, dst, 4096, t)
    assert np.array_equal(dst.view(np.uint32), oracle_mod.dequantize(t, blocks, 4096).view(np.uint32))


@pytest.mark.parametrize("fmt,K", [("Q4_0", 96), ("Q4_0", 288), ("Q8_0", 288), ("Q8_0", 32), ("Q4_K", 768)])
def test_k_not_multiple_of_64_elements(cuda, oracle_mod, fmt, K):
    """Activation rows that end in a partial 128-byte line of shared memory."""
    t = synth.IDS[fmt]
    N = 211
    blocks = synth.random_blocks(t, N, K, seed=800 + K)
    X = synth.random_activations(3, K, seed=801)
    got = _gemm_gpu(cuda, t, blocks, X, N, K)
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, 3, N, K)) <= REL_L2_TOL


def test_unaligned_activation_pointer(cuda, oracle_mod):
    """X starting 4 bytes past a 16-byte boundary: scalar activation loads."""
    torch = cuda
    t = synth.Q5_K
    N, K, M = 333, 1024, 2
    blocks = synth.random_blocks(t, N, K, seed=900)
    X = synth.random_activations(M, K, seed=901)
    d_w = torch.from_numpy(blocks.reshape(-1)).cuda()
    d_xbuf = torch.zeros(M * K + 4, dtype=torch.float32, device="cuda")
    d_xbuf[1:1 + M * K] = torch.from_numpy(X.reshape(-1)).cuda()
    d_y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    swq.gemm(t, d_w, d_xbuf.data_ptr() + 4, d_y, M, N, K)
    swq.check()
    assert rel_l2(d_y.cpu().numpy(), oracle_mod.gemm(t, blocks, X, M, N, K)) <= REL_L2_TOL


@pytest.mark.parametrize("fmt", ["Q6_K", "Q4_K", "Q8_0", "Q5_K"])
@pytest.mark.parametrize("M", [1, 2])
def test_llama_down_proj_shape(cuda, oracle_mod, fmt, M):
    """N=4096, K=14336 (Llama-3-8B FFN down-projection): rows split along K."""
    t = synth.IDS[fmt]
    N, K = 4096, 14336
    blocks = synth.random_blocks(t, N, K, seed=1000 + t)
    X = synth.random_activations(M, K, seed=1001)
    got = _gemm_gpu(cuda, t, blocks, X, N, K)
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, M, N, K)) <= REL_L2_TOL


@pytest.mark.parametrize("fmt,N,K", [("Q4_K", 600, 3072), ("Q4_K", 333, 2048), ("Q4_0", 901, 4096),
                                      ("Q8_0", 517, 8192), ("Q4_K", 700, 512), ("Q6_K", 257, 1024)])
def test_whole_row_work_splits(cuda, oracle_mod, fmt, N, K):
    """Row widths whose unit counts do (64, 128, 8, 16) and do not (48) divide
    the consumer lanes, and several row groups per CTA."""
    t = synth.IDS[fmt]
    blocks = synth.random_blocks(t, N, K, seed=1100 + K)
    X = synth.random_activations(1, K, seed=1101)
    got = _gemm_gpu(cuda, t, blocks, X, N, K)
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, 1, N, K)) <= REL_L2_TOL


@pytest.mark.parametrize("smem_kb,stage_kb,ctas", [(220, 0, 0), (220, 24, 0), (0, 16, 0), (100, 40, 0), (0, 0, 2), (0, 32, 2)])
@pytest.mark.parametrize("fmt,N,K", [("Q4_K", 28672, 4096), ("Q6_K", 4096, 14336), ("Q6_K", 1000, 4096),
                                      ("Q4_K", 333, 2048)])
def test_ring_options(cuda, oracle_mod, smem_kb, stage_kb, ctas, fmt, N, K):
    """Other weight-ring shapes (SWQ_OPT_GEMV_SMEM_KB / SWQ_OPT_GEMV_STAGE_KB /
    SWQ_OPT_GEMV_CTAS_PER_SM): whole-row and row-chunk stages, groups shorter
    than a stage, two CTAs per SM."""
    t = synth.IDS[fmt]
    blocks = synth.random_blocks(t, N, K, seed=N + K)
    X = synth.random_activations(1, K, seed=K)
    swq.set_option(swq.OPT_GEMV_SMEM_KB, smem_kb)
    swq.set_option(swq.OPT_GEMV_STAGE_KB, stage_kb)
    swq.set_option(swq.OPT_GEMV_CTAS_PER_SM, ctas)
    try:
        got = _gemm_gpu(cuda, t, blocks, X, N, K)
    finally:
        swq.set_option(swq.OPT_GEMV_SMEM_KB, 0)
        swq.set_option(swq.OPT_GEMV_STAGE_KB, 0)
        swq.set_option(swq.OPT_GEMV_CTAS_PER_SM, 0)
    assert rel_l2(got, oracle_mod.gemm(t, blocks, X, 1, N, K)) <= REL_L2_TOL


@pytest.mark.parametrize("fp32,int_mma", [(1, 0), (1, 1), (1, 2), (0, 0)],
                         ids=["fp32", "fp32+intmma-q6k", "fp32+intmma-all", "int16"])
@pytest.mark.parametrize("fmt,N,K", [("Q4_K", 300, 4096), ("Q6_K", 333, 4096), ("Q6_K", 64, 14336),
                                     ("Q4_K", 37, 1024), ("Q4_K", 1, 256), ("Q6_K", 17, 2048)])
def test_gemv_forms(cuda, oracle_mod, fp32, int_mma, fmt, N, K):
    """Every single-row form against the oracle: fp32 activations with and
    without the integer tensor-core dot products, and 16-bit fixed-point
    activations; rows not a multiple of the 16-row tile, K below and above a
    chunk, K that the tensor-core form does not take (Q6_K 1024 is not a
    multiple of 2048: the fp32 form serves it)."""
    t = synth.IDS[fmt]
    blocks = synth.random_blocks(t, N, K, seed=900 + N)
    X = synth.random_activations(1, K, seed=901)
    swq.set_option(swq.OPT_GEMV_FP32_ACT, fp32)
    swq.set_option(swq.OPT_GEMV_INT_MMA, int_mma)
    try:
        got = _gemm_gpu(cuda, t, blocks, X, N, K)
    finally:
        swq.set_option(swq.OPT_GEMV_FP32_ACT, 1)
        swq.set_option(swq.OPT_GEMV_INT_MMA, 2)
    want = oracle_mod.gemm(t, blocks, X, 1, N, K)
    tol = 1e-5 if fp32 else REL_L2_TOL  # fp32 forms: rounding of fp32 sums only
    assert rel_l2(got, want) <= tol


@pytest.mark.parametrize("int_mma", [1, 2])
@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_int_mma_dynamic_range(cuda, oracle_mod, int_mma, fmt):
    """Activations over twelve decades (each 16/32-element part gets its own
    fixed-point scale), a part of zeros and a part of subnormals: the integer
    tensor-core form stays at fp32 accuracy."""
    t = synth.IDS[fmt]
    N, K = 96, 4096
    blocks = synth.random_blocks(t, N, K, seed=950)
    rng = np.random.default_rng(951)
    x = (rng.standard_normal(K) * 10.0 ** rng.uniform(-6, 6, K)).astype(np.float32)
    x[64:96] = 0.0
    x[128:144] = np.float32(1e-40)
    X = x.reshape(1, K)
    swq.set_option(swq.OPT_GEMV_INT_MMA, int_mma)
    try:
        got = _gemm_gpu(cuda, t, blocks, X, N, K)
    finally:
        swq.set_option(swq.OPT_GEMV_INT_MMA, 2)
    want = oracle_mod.gemm(t, blocks, X, 1, N, K)
    assert rel_l2(got, want) <= 1e-5
