"""swq_gemm_noalloc, the allocation-free form of swq_gemm.

Some callers cannot let a library allocate GPU memory: a serving engine that
hands all free HBM to its KV cache at start-up, or a process whose caching
allocator owns every device byte.  swq_gemm_noalloc keeps its scratch in fixed
device arrays inside libswq instead of taking it from a memory pool.

The GPU test calls it through the C ABI (ctypes, libswq.so), three calls in a
row on the same fixed arrays.  Each result is compared with swq_gemm's on the
same inputs and with the oracle (the reference's CPU routine), within the
GEMM tests' relative-L2 tolerance:
  1. Q4_K M=300 N=1000 K=4096: split-K in 8 parts, the same plan as swq_gemm,
     so the output is bit-identical to swq_gemm's;
  2. Q6_K M=40 N=384 K=2048: a smaller M x K over arrays that still hold the
     first call's activations, split in 4, bit-identical again;
  3. Q4_K M=256 N=9472 K=4096: swq_gemm splits K in 2, but 2 x M x N partial
     products do not fit the fixed partials array, so this call runs unsplit
     (a different summation order: compared within tolerance).
This file is collected last, so a run that stops at the first failure has
run every other test first.
"""
import numpy as np
import pytest

import swq
from conftest import REL_L2_TOL, rel_l2
from swq import synth

# (format, M, N, K, bit-identical to swq_gemm)
CASES = [("Q4_K", 300, 1000, 4096, True), ("Q6_K", 40, 384, 2048, True), ("Q4_K", 256, 9472, 4096, False)]


def _call(L, t, w, x, y, M, N, K, stream):
    return L.swq_gemm_noalloc(t, w.data_ptr(), x.data_ptr(), y.data_ptr(), M, N, K, stream)


@pytest.mark.gpu
def test_noalloc_matches_gemm(cuda, oracle_mod):
    torch = cuda
    L = swq.lib()
    stream = int(torch.cuda.current_stream().cuda_stream)
    for i, (fmt, M, N, K, same_plan) in enumerate(CASES):
        t = synth.IDS[fmt]
        blocks = synth.random_blocks(t, N, K, seed=3000 + i)
        X = synth.random_activations(M, K, seed=3100 + i)
        w = torch.from_numpy(blocks.reshape(-1)).cuda()
        x = torch.from_numpy(X).cuda()
        y_ref = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        swq.gemm(t, w, x, y_ref, M, N, K)
        assert _call(L, t, w, x, y, M, N, K, stream) == swq.Status.OK, L.swq_last_error()
        swq.check()
        got, want = y.cpu().numpy(), y_ref.cpu().numpy()
        assert np.all(np.isfinite(got)), fmt
        if same_plan:
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (fmt, M, N, K)
        else:
            assert rel_l2(got, want) <= REL_L2_TOL
        assert rel_l2(got, oracle_mod.gemm(t, blocks, X, M, N, K)) <= REL_L2_TOL, (fmt, M, N, K)


def test_noalloc_rejects_oversize():
    """M * K above the fixed scratch is refused before any device work."""
    L = swq.lib()
    K = 4096
    M = swq.GEMM_NOALLOC_MAX_X_ELEMS // K + 1
    rc = L.swq_gemm_noalloc(swq.Q4_K, 16, 16, 16, M, 128, K, None)
    assert rc == swq.Status.BAD_SHAPE
    assert b"exceeds its fixed scratch" in L.swq_last_error()
