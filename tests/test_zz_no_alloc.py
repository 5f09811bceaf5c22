"""swq_gemm_noalloc, the allocation-free form of swq_gemm.

The GPU test calls it through the C ABI (ctypes, libswq.so) and compares its
output with swq_gemm's on the same inputs, within the relative-L2 tolerance
of the other GEMM tests, on two calls in a row.  The second call has another
format and a smaller M x K, so it runs over the fixed scratch array while that
still holds the first call's activations.
"""
import numpy as np
import pytest

import swq
from conftest import REL_L2_TOL, rel_l2
from swq import synth


def _call(L, t, w, x, y, M, N, K, stream):
    return L.swq_gemm_noalloc(t, w.data_ptr(), x.data_ptr(), y.data_ptr(), M, N, K, stream)


@pytest.mark.gpu
def test_noalloc_matches_gemm(cuda):
    torch = cuda
    L = swq.lib()
    stream = int(torch.cuda.current_stream().cuda_stream)
    cases = [("Q4_K", 300, 1000, 4096), ("Q6_K", 40, 384, 2048)]
    for i, (fmt, M, N, K) in enumerate(cases):
        t = synth.IDS[fmt]
        w = torch.from_numpy(synth.random_blocks(t, N, K, seed=3000 + i).reshape(-1)).cuda()
        x = torch.from_numpy(synth.random_activations(M, K, seed=3100 + i)).cuda()
        y_ref = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        swq.gemm(t, w, x, y_ref, M, N, K)
        assert _call(L, t, w, x, y, M, N, K, stream) == swq.Status.OK, L.swq_last_error()
        swq.check()
        got, want = y.cpu().numpy(), y_ref.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert rel_l2(got, want) <= REL_L2_TOL


def test_noalloc_rejects_oversize():
    """M * K above the fixed scratch is refused before any device work."""
    L = swq.lib()
    K = 4096
    M = swq.GEMM_NOALLOC_MAX_X_ELEMS // K + 1
    rc = L.swq_gemm_noalloc(swq.Q4_K, 16, 16, 16, M, 128, K, None)
    assert rc == swq.Status.BAD_SHAPE
    assert b"exceeds its fixed scratch" in L.swq_last_error()
