"""MoE grouped expert GEMM (swq_grouped_gemm) against the oracle, expert by expert.

The reference has no MoE path; each expert's rows are checked against the
oracle's per-row reference product (one Compute::matmul_transposed_q per row,
src/tensor.h:1212) with that expert's weights.  Tolerance: relative L2 <= 1e-3
per expert, as for swq_gemm.
"""
import numpy as np
import pytest

import swq
from conftest import REL_L2_TOL, rel_l2
from swq import synth

pytestmark = pytest.mark.gpu


def _run(torch, oracle_mod, t, counts, N, K, seed, offsets_bytes=None, fn=None):
    """Experts with `counts[e]` rows each; returns per-expert rel-L2 and the
    rows outside every expert (must stay NaN)."""
    E = len(counts)
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    rows = int(offs[-1])
    blocks = [synth.random_blocks(t, N, K, seed=seed + e) for e in range(E)]
    X = synth.random_activations(max(rows, 1), K, seed=seed + 1000)[:rows]
    # every expert's blocks in one allocation, optionally at odd byte offsets
    wb = synth.matrix_bytes(t, N, K)
    pad = [0 if offsets_bytes is None else offsets_bytes[e % len(offsets_bytes)] for e in range(E)]
    starts, pos = [], 0
    for e in range(E):
        pos += pad[e]
        starts.append(pos)
        pos += wb
    buf = torch.zeros(pos + 64, dtype=torch.uint8, device="cuda")
    for e in range(E):
        buf[starts[e]:starts[e] + wb] = torch.from_numpy(blocks[e].reshape(-1)).cuda()
    ptrs = torch.tensor([buf.data_ptr() + st for st in starts], dtype=torch.int64, device="cuda")
    d_off = torch.from_numpy(offs).cuda()
    d_x = torch.from_numpy(np.ascontiguousarray(X, dtype=np.float32)).cuda() if rows else \
        torch.zeros((1, K), dtype=torch.float32, device="cuda")
    d_y = torch.full((max(rows, 1), N), float("nan"), dtype=torch.float32, device="cuda")
    (fn or swq.grouped_gemm)(t, ptrs, d_off, d_x, d_y, E, rows, N, K)
    swq.check()
    Y = d_y.cpu().numpy()
    errs = []
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        if b > a:
            want = oracle_mod.gemm(t, blocks[e], X[a:b], b - a, N, K)
            errs.append(rel_l2(Y[a:b], want))
    return errs


@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"])
def test_prefill_routing(cuda, oracle_mod, fmt):
    """Expert gate/up shape (N=512, K=2048), ~32 rows per expert with empty experts."""
    rng = np.random.default_rng(11)
    counts = rng.integers(0, 70, size=12)
    counts[3] = 0
    counts[7] = 0
    errs = _run(cuda, oracle_mod, synth.IDS[fmt], counts, 512, 2048, seed=4000)
    assert max(errs) <= REL_L2_TOL, errs


def test_decode_routing(cuda, oracle_mod):
    """Decode: 1-2 rows per expert, most experts empty (64 experts)."""
    rng = np.random.default_rng(12)
    counts = np.where(rng.random(64) < 0.4, rng.integers(1, 3, size=64), 0)
    errs = _run(cuda, oracle_mod, synth.Q4_K, counts, 512, 2048, seed=4100)
    assert errs and max(errs) <= REL_L2_TOL


def test_down_projection_shape(cuda, oracle_mod):
    """Expert down projection: N=2048, K=512; one expert with many token tiles."""
    counts = [5, 300, 0, 40, 129]
    errs = _run(cuda, oracle_mod, synth.Q6_K, counts, 2048, 512, seed=4200)
    assert max(errs) <= REL_L2_TOL


def test_wide_experts(cuda, oracle_mod):
    """Mean rows per expert above 128: the 256-token tile."""
    errs = _run(cuda, oracle_mod, synth.Q4_K, [260, 0, 300], 384, 1024, seed=4300)
    assert max(errs) <= REL_L2_TOL


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K", "Q8_0", "Q4_0"])
def test_unaligned_expert_weights(cuda, oracle_mod, fmt):
    """Expert matrices at 1-, 2-, 6- and 10-byte offsets inside one buffer."""
    errs = _run(cuda, oracle_mod, synth.IDS[fmt], [17, 33, 64, 3], 256, 1024, seed=4400,
                offsets_bytes=[1, 2, 6, 10])
    assert max(errs) <= REL_L2_TOL


def test_one_expert_equals_gemm(cuda):
    """A single expert covering every row is the dense GEMM, bit for bit (80
    output tiles: the dense call does not split K, so both sum in one order)."""
    torch = cuda
    t, N, K, M = synth.Q4_K, 10240, 1024, 200
    w = torch.from_numpy(synth.random_blocks(t, N, K, seed=4500).reshape(-1)).cuda()
    x = torch.from_numpy(synth.random_activations(M, K, seed=4501)).cuda()
    y1 = torch.empty((M, N), dtype=torch.float32, device="cuda")
    y2 = torch.empty((M, N), dtype=torch.float32, device="cuda")
    swq.gemm(t, w, x, y1, M, N, K)
    ptrs = torch.tensor([w.data_ptr()], dtype=torch.int64, device="cuda")
    offs = torch.tensor([0, M], dtype=torch.int32, device="cuda")
    swq.grouped_gemm(t, ptrs, offs, x, y2, 1, M, N, K)
    swq.check()
    assert torch.equal(y1, y2)


def test_rows_outside_experts_untouched(cuda):
    """Offsets that stop short of total_rows: the remaining rows keep their value."""
    torch = cuda
    t, N, K = synth.Q4_K, 256, 512
    w = torch.from_numpy(synth.random_blocks(t, N, K, seed=4600).reshape(-1)).cuda()
    x = torch.from_numpy(synth.random_activations(40, K, seed=4601)).cuda()
    y = torch.full((40, N), 7.0, dtype=torch.float32, device="cuda")
    ptrs = torch.tensor([w.data_ptr(), w.data_ptr()], dtype=torch.int64, device="cuda")
    offs = torch.tensor([0, 10, 25], dtype=torch.int32, device="cuda")
    swq.grouped_gemm(t, ptrs, offs, x, y, 2, 40, N, K)
    swq.check()
    assert torch.all(y[25:] == 7.0)
    assert torch.all(torch.isfinite(y[:25]))


# ---------------------------------------------------------------- grouped GEMV
@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"])
def test_grouped_gemv_decode_routing(cuda, oracle_mod, fmt):
    """swq_grouped_gemv: 1-2 rows per expert, most of 64 experts empty."""
    rng = np.random.default_rng(13)
    counts = np.where(rng.random(64) < 0.4, rng.integers(1, 3, size=64), 0)
    errs = _run(cuda, oracle_mod, synth.IDS[fmt], counts, 512, 2048, seed=4700, fn=swq.grouped_gemv)
    assert errs and max(errs) <= REL_L2_TOL, errs


@pytest.mark.parametrize("counts", [[9, 0, 1, 5, 0, 3], [4, 4, 4, 4], [1] * 40])
def test_grouped_gemv_rows_per_expert(cuda, oracle_mod, counts):
    """More rows per expert than one pass holds (groups of 1, 2 or 4 rows), and
    the expert down-projection shape (N=2048, K=512)."""
    errs = _run(cuda, oracle_mod, synth.Q4_K, counts, 2048, 512, seed=4800, fn=swq.grouped_gemv)
    assert max(errs) <= REL_L2_TOL, errs


def test_grouped_gemv_matches_grouped_gemm(cuda, oracle_mod):
    """The GEMV and tensor-core grouped paths agree within the GEMM tolerance."""
    rng = np.random.default_rng(14)
    counts = rng.integers(0, 3, size=32)
    e1 = _run(cuda, oracle_mod, synth.Q6_K, counts, 640, 1024, seed=4900, fn=swq.grouped_gemv)
    e2 = _run(cuda, oracle_mod, synth.Q6_K, counts, 640, 1024, seed=4900)
    assert max(e1) <= REL_L2_TOL and max(e2) <= REL_L2_TOL


def test_grouped_gemv_misaligned_expert_reported(cuda):
    """An expert matrix off a 16-byte boundary is skipped (its rows keep their
    value) and swq_check reports it; the aligned experts are computed."""
    torch = cuda
    t, N, K = synth.Q4_K, 256, 512
    wb = synth.matrix_bytes(t, N, K)
    buf = torch.zeros(2 * wb + 64, dtype=torch.uint8, device="cuda")
    blocks = synth.random_blocks(t, N, K, seed=5000)
    buf[:wb] = torch.from_numpy(blocks.reshape(-1)).cuda()
    buf[wb + 2:2 * wb + 2] = torch.from_numpy(blocks.reshape(-1)).cuda()
    ptrs = torch.tensor([buf.data_ptr(), buf.data_ptr() + wb + 2], dtype=torch.int64, device="cuda")
    offs = torch.tensor([0, 3, 6], dtype=torch.int32, device="cuda")
    x = torch.from_numpy(synth.random_activations(6, K, seed=5001)).cuda()
    y = torch.full((6, N), 7.0, dtype=torch.float32, device="cuda")
    swq.grouped_gemv(t, ptrs, offs, x, y, 2, 6, N, K)
    with pytest.raises(swq.SwqError):
        swq.check()
    swq.check()  # the status was cleared by the check that reported it
    assert torch.all(y[3:] == 7.0)
    assert torch.all(torch.isfinite(y[:3])) and not torch.all(y[:3] == 7.0)
