"""The arithmetic of the Q4_K / Q6_K GEMV kernels, restated in numpy on the
CPU, against the oracle restatement of cpu_matmul_transposed_q4_k / _q6_k
(src/tensor.h:769-856): the batched K-quant GEMV (gemv_kqm.cu, 2..32 rows)
first, the single-row integer GEMV (gemv_kq.cu) at the end.

The kernel holds each activation row per 256-element super-block as
x 2^(14 - E) = h + l, two fp16 numbers (E: the block's largest binary
exponent), multiplies them by exact fp16 weight operands (Q4_K: q sc; Q6_K:
q - 32) and sums in fp32; the Q4_K mins multiply the sub-block sums of the
scaled x (times 2^-5, split the same way).  Here the same representation is
built with the kernel's roundings (prep_kernel: fp32 scaling, round-to-nearest
fp16, the sums of 32 in the kernel's addition tree) and the products are summed
in float64, which isolates the representation's error from the fp32 sums:

* against the exact sum of the reference's own fp32 weights it stays near
  5e-8 (relative L2 per row), far below the reference's own fp32 rounding
  (about 1e-6 to 3e-6 from the exact sum on these shapes);
* so against the oracle it is within the 1e-5 the GPU tests hold the kernel
  to (tests/test_gpu_gemv_kqm.py), with room for the kernel's fp32 sums.

The Q4_K / Q6_K block decoders below follow the GGUF layouts
(src/tensor.h:218-227, 329-358, 398-432) and are pinned bit for bit to the
oracle's dequantization first."""
import numpy as np
import pytest

from conftest import rel_l2
from swq import synth

F16, F32, F64 = np.float16, np.float32, np.float64
Q4_K, Q6_K = synth.IDS["Q4_K"], synth.IDS["Q6_K"]
GPU_TOL = 1e-5   # the kernel's bound against the oracle (GPU tests)
REPR_TOL = 3e-7  # the representation alone, against the exact sum


def _f16(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b).view(F16)[..., 0].astype(F32)


def q4k_parts(blocks, N, K):
    """d, dmin [N, nb]; 6-bit scales and mins [N, nb, 8]; nibbles q [N, nb, 256]
    with element 64 g + 32 hi + l in sub-block 2 g + hi."""
    nb = K // 256
    B = blocks.reshape(N, nb, 144)
    d, dmin = _f16(B[:, :, 0:2]), _f16(B[:, :, 2:4])
    s = B[:, :, 4:16].astype(np.int32)
    sc = np.empty((N, nb, 8), np.int32)
    mn = np.empty((N, nb, 8), np.int32)
    for j in range(4):
        sc[..., j], mn[..., j] = s[..., j] & 63, s[..., j + 4] & 63
        sc[..., j + 4] = (s[..., j + 8] & 15) | ((s[..., j] >> 6) << 4)
        mn[..., j + 4] = (s[..., j + 8] >> 4) | ((s[..., j + 4] >> 6) << 4)
    qs = B[:, :, 16:144].astype(np.int32).reshape(N, nb, 4, 1, 32)
    q = np.concatenate([qs & 15, qs >> 4], axis=3).reshape(N, nb, 256)
    return d, dmin, sc, mn, q


def q6k_parts(blocks, N, K):
    """d [N, nb]; int8 scales [N, nb, 16] (sub-block of 16 = element // 16);
    q - 32 [N, nb, 256]."""
    nb = K // 256
    B = blocks.reshape(N, nb, 210)
    ql, qh = B[:, :, 0:128].astype(np.int32), B[:, :, 128:192].astype(np.int32)
    sc = B[:, :, 192:208].view(np.int8).astype(np.int32)
    d = _f16(B[:, :, 208:210])
    q = np.empty((N, nb, 256), np.int32)
    for n in range(2):
        lo, hi = ql[:, :, 64 * n:64 * n + 32], ql[:, :, 64 * n + 32:64 * n + 64]
        h = qh[:, :, 32 * n:32 * n + 32]
        base = 128 * n
        q[:, :, base:base + 32] = (lo & 15) | ((h & 3) << 4)
        q[:, :, base + 32:base + 64] = (hi & 15) | (((h >> 2) & 3) << 4)
        q[:, :, base + 64:base + 96] = (lo >> 4) | (((h >> 4) & 3) << 4)
        q[:, :, base + 96:base + 128] = (hi >> 4) | (((h >> 6) & 3) << 4)
    return d, sc, q - 32


def dequant_f32(t, blocks, N, K):
    """The reference's fp32 weights from the decoded parts, in its expression
    order: Q4_K (d sc) q - dmin m; Q6_K (d sc) q."""
    if t == Q4_K:
        d, dmin, sc, mn, q = q4k_parts(blocks, N, K)
        d1 = (d[..., None] * np.repeat(sc, 32, axis=2).astype(F32)).astype(F32)
        m1 = (dmin[..., None] * np.repeat(mn, 32, axis=2).astype(F32)).astype(F32)
        return (d1 * q.astype(F32) - m1).astype(F32).reshape(N, K)
    d, sc, q = q6k_parts(blocks, N, K)
    d1 = (d[..., None] * np.repeat(sc, 16, axis=2).astype(F32)).astype(F32)
    return (d1 * q.astype(F32)).astype(F32).reshape(N, K)


def split_row(x: np.ndarray, nb: int):
    """prep_kernel for one activation row: per super-block h, l (fp16 values),
    the Q4_K mins' B operand h', l' (sub-block sums of 32 times 2^-5) and the
    scale 2^(E - 14)."""
    x = np.asarray(x, F32).reshape(nb, 256)
    mx = np.abs(x).max(axis=1).astype(F32)
    E = np.maximum(((mx.view(np.int32) >> 23) & 0xFF) - 126, -100)
    u = (x * np.ldexp(F32(1), 14 - E).astype(F32)[:, None]).astype(F32)
    h = u.astype(F16)
    l = (u - h.astype(F32)).astype(F16)
    v = u.reshape(nb, 8, 4, 8)  # sub-block of 32, lane, its 8 elements
    lane = ((v[..., 0] + v[..., 1]) + (v[..., 2] + v[..., 3])) + ((v[..., 4] + v[..., 5]) + (v[..., 6] + v[..., 7]))
    s32 = ((lane[..., 0] + lane[..., 1]) + (lane[..., 2] + lane[..., 3])).astype(F32)
    xp = (s32 * F32(0.03125)).astype(F32)
    hp = xp.astype(F16)
    lp = (xp - hp.astype(F32)).astype(F16)
    return h, l, hp, lp, np.ldexp(1.0, E - 14)


def emulate(t, blocks, X, N, K) -> np.ndarray:
    """Y[M, N] from the kernel's representation, products and sums in float64."""
    M, nb = X.shape[0], K // 256
    Y = np.zeros((M, N))
    if t == Q4_K:
        d, dmin, sc, mn, q = q4k_parts(blocks, N, K)
        A = (q * np.repeat(sc, 32, axis=2)).astype(F64)  # q sc: the fp16 A operand
        for m in range(M):
            h, l, hp, lp, xs = split_row(X[m], nb)
            C = np.einsum("nbk,bk->nb", A, h.astype(F64) + l.astype(F64))
            Cm = np.einsum("nbj,bj->nb", mn.astype(F64), hp.astype(F64) + lp.astype(F64))
            Y[m] = ((d.astype(F64) * C - 32.0 * dmin.astype(F64) * Cm) * xs[None, :]).sum(axis=1)
        return Y
    d, sc, q = q6k_parts(blocks, N, K)
    A = q.reshape(N, nb, 16, 16).astype(F64)  # q - 32: the fp16 A operand
    for m in range(M):
        h, l, _, _, xs = split_row(X[m], nb)
        Cj = np.einsum("nbjk,bjk->nbj", A, (h.astype(F64) + l.astype(F64)).reshape(nb, 16, 16))
        Y[m] = (d.astype(F64) * (sc * Cj).sum(axis=2) * xs[None, :]).sum(axis=1)
    return Y


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_decoders_match_oracle_dequant(oracle_mod, fmt):
    t = synth.IDS[fmt]
    N, K = 96, 2048
    blocks = synth.random_blocks(t, N, K, seed=5)
    want = oracle_mod.dequantize(t, blocks, N * K).reshape(N, K)
    got = dequant_f32(t, blocks, N, K)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_operands_are_exact(fmt):
    """Every A operand is an integer fp16 holds exactly, so each product with
    an fp16 h or l is exact in the MMA's fp32 (at most 11 + 11 bits)."""
    t = synth.IDS[fmt]
    N, K = 64, 2048
    blocks = synth.random_blocks(t, N, K, seed=6)
    if t == Q4_K:
        _, _, sc, mn, q = q4k_parts(blocks, N, K)
        A = q * np.repeat(sc, 32, axis=2)
        assert A.max() <= 945 and A.min() >= 0 and mn.max() <= 63
        ops = [A, mn]
    else:
        _, _, q = q6k_parts(blocks, N, K)
        assert q.min() >= -32 and q.max() <= 31
        ops = [q]
    for a in ops:
        assert np.array_equal(a.astype(F16).astype(np.int64), a)
    h, l, _, _, _ = split_row(synth.random_activations(1, K, seed=7)[0], K // 256)
    a = ops[0].reshape(-1, K // 256, 256)[:4].astype(F32)
    for part in (h, l):
        prod32 = a * part.astype(F32)[None]
        assert np.array_equal(prod32.astype(F64), a.astype(F64) * part.astype(F64)[None])


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("N,K,M", [(256, 4096, 4), (128, 14336, 2), (64, 2048, 9)])
def test_representation_within_kernel_bound(oracle_mod, fmt, N, K, M):
    t = synth.IDS[fmt]
    blocks = synth.random_blocks(t, N, K, seed=N + K)
    X = synth.random_activations(M, K, seed=K + M)
    ref = np.asarray(oracle_mod.gemm(t, blocks, X, M, N, K)).reshape(M, N)
    exact = X.astype(F64) @ dequant_f32(t, blocks, N, K).astype(F64).T
    emu = emulate(t, blocks, X, N, K)
    for m in range(M):
        assert rel_l2(emu[m], exact[m]) <= REPR_TOL, (m, rel_l2(emu[m], exact[m]))
        assert rel_l2(emu[m], ref[m]) <= GPU_TOL, (m, rel_l2(emu[m], ref[m]))


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_representation_edge_rows(oracle_mod, fmt):
    """A zero row, a row whose super-blocks differ by 1e40 in scale, one with
    1e30 beside 1e-30 and a block of 1e-30, and a row of normal magnitude with
    a super-block of fp32 subnormals: per-block scaling keeps every block's own
    22 bits, and a subnormal block adds nothing measurable to a normal row."""
    t = synth.IDS[fmt]
    N, K = 64, 2048
    nb = K // 256
    blocks = synth.random_blocks(t, N, K, seed=11)
    base = synth.random_activations(1, K, seed=12)[0].astype(F32)
    rows = [np.zeros(K, F32)]
    r = base.copy()
    for b in range(nb):
        r[256 * b:256 * b + 256] *= F32(10.0 ** (20 if b % 2 else -20))
    rows.append(r)
    r = base.copy()
    r[3], r[700] = F32(1e30), F32(-3e29)
    r[256:512] *= F32(1e-30)
    rows.append(r)
    r = base.copy()
    r[1024:1280] = F32(1e-40)  # a super-block of fp32 subnormals
    rows.append(r)
    X = np.stack(rows).astype(F32)
    ref = np.asarray(oracle_mod.gemm(t, blocks, X, X.shape[0], N, K)).reshape(X.shape[0], N)
    exact = X.astype(F64) @ dequant_f32(t, blocks, N, K).astype(F64).T
    emu = emulate(t, blocks, X, N, K)
    assert np.array_equal(emu[0], np.zeros(N))
    for m in range(1, X.shape[0]):
        if np.linalg.norm(exact[m]) == 0:
            continue
        assert rel_l2(emu[m], exact[m]) <= REPR_TOL, (m, rel_l2(emu[m], exact[m]))
        assert rel_l2(emu[m], ref[m]) <= GPU_TOL, (m, rel_l2(emu[m], ref[m]))


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_rows_below_the_block_floor(oracle_mod, fmt):
    """The kernel's scale factors 2^(14 - E) and 2^(E - 14) stay normal fp32
    numbers (E >= -100), so a super-block whose largest element is below
    2^-117 (about 6e-36; its low fp16 part turns subnormal) keeps fewer than
    22 bits.  Whole rows that small: at 2^-110 nothing is lost; at the bottom
    of fp32's normal range (largest element about 3e-38) the row stays within
    3e-4 of the exact sum, inside the 1e-3 matmul tolerance; a row of fp32
    subnormals (about 3e-40) does not (about 7e-3), where the reference's own
    fp32 loop stays near 1e-6.  Activations of a model never sit there."""
    t = synth.IDS[fmt]
    N, K = 64, 2048
    blocks = synth.random_blocks(t, N, K, seed=13)
    W = dequant_f32(t, blocks, N, K).astype(F64)
    base = synth.random_activations(1, K, seed=14)[0].astype(F32)
    for scale, bound in ((2.0 ** -110, REPR_TOL), (1e-38, 3e-4), (1e-40, 2e-2)):
        X = (base * F32(scale)).astype(F32)[None]
        exact = X.astype(F64) @ W.T
        ref = np.asarray(oracle_mod.gemm(t, blocks, X, 1, N, K)).reshape(1, N)
        err = rel_l2(emulate(t, blocks, X, N, K)[0], exact[0])
        assert err <= bound, (scale, err)
        assert rel_l2(ref[0], exact[0]) <= 1e-5


# ---------------------------------------------------------------------------
# Single-row integer GEMV (gemv_kq.cu): per 256-element super-block,
# Z = round(x 2^(30 - E)) (E: the block's largest binary exponent, E >= -96)
# split into int8 limbs; the sub-block sums S_j = sum q_k Z_k are exact
# integers, scaled by 2^(E - 30) once per super-block; the sums X_j of x for
# the Q4_K mins and the Q6_K offset are fp32 sums in the kernel's tree.  The
# emulation keeps the integers exact and sums the rest in float64.

def kq_split_row(x: np.ndarray, nb: int, t: int):
    x = np.asarray(x, F32).reshape(nb, 256)
    mx = np.abs(x).max(axis=1).astype(F32)
    E = np.maximum(((mx.view(np.int32) >> 23) & 0xFF) - 126, -96)
    Z = np.rint((x * np.ldexp(F32(1), 30 - E).astype(F32)[:, None]).astype(F32).astype(F64)).astype(np.int64)
    if t == Q4_K:  # sub-blocks of 32: four lanes of 8, (l0 + l1) + (l2 + l3)
        v = x.reshape(nb, 8, 4, 8)
        lane = ((v[..., 0] + v[..., 1]) + (v[..., 2] + v[..., 3])) + ((v[..., 4] + v[..., 5]) + (v[..., 6] + v[..., 7]))
        Xj = ((lane[..., 0] + lane[..., 1]) + (lane[..., 2] + lane[..., 3])).astype(F32)
    else:  # sub-blocks of 16: two lanes of 8
        v = x.reshape(nb, 16, 2, 8)
        lane = ((v[..., 0] + v[..., 1]) + (v[..., 2] + v[..., 3])) + ((v[..., 4] + v[..., 5]) + (v[..., 6] + v[..., 7]))
        Xj = (lane[..., 0] + lane[..., 1]).astype(F32)
    return Z, Xj, np.ldexp(1.0, E - 30)


def emulate_kq(t, blocks, x, N, K) -> np.ndarray:
    """y[N] of the single-row kernel's representation (exact integer sums)."""
    nb = K // 256
    Z, Xj, xe = kq_split_row(x, nb, t)
    if t == Q4_K:
        d, dmin, sc, mn, q = q4k_parts(blocks, N, K)
        S = (q.astype(np.int64) * Z[None]).reshape(N, nb, 8, 32).sum(axis=3)
        I = (sc.astype(np.int64) * S).sum(axis=2)
        mins = (mn * Xj[None].astype(F64)).sum(axis=2)
        return (d.astype(F64) * I.astype(F64) * xe[None] - dmin.astype(F64) * mins).sum(axis=1)
    d, sc, qm = q6k_parts(blocks, N, K)
    S = ((qm + 32).astype(np.int64) * Z[None]).reshape(N, nb, 16, 16).sum(axis=3)
    I = (sc.astype(np.int64) * S).sum(axis=2)
    off = 32.0 * (sc * Xj[None].astype(F64)).sum(axis=2)
    return (d.astype(F64) * (I.astype(F64) * xe[None] - off)).sum(axis=1)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("N,K", [(256, 4096), (128, 14336)])
def test_single_row_representation(oracle_mod, fmt, N, K):
    """30-bit fixed point per super-block with exact integer sums: about 1e-8
    (Q4_K) to 1e-7 (Q6_K) from the exact sum of the reference's fp32 weights,
    an order of magnitude under the reference's own fp32 loop."""
    t = synth.IDS[fmt]
    blocks = synth.random_blocks(t, N, K, seed=N + 2 * K)
    x = synth.random_activations(1, K, seed=K + 1)[0]
    exact = dequant_f32(t, blocks, N, K).astype(F64) @ x.astype(F64)
    ref = np.asarray(oracle_mod.gemv(t, blocks, x, N, K))
    emu = emulate_kq(t, blocks, x, N, K)
    assert rel_l2(emu, exact) <= REPR_TOL
    assert rel_l2(emu, ref) <= GPU_TOL


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_single_row_below_the_block_floor(oracle_mod, fmt):
    """E >= -96 keeps the single-row kernel's scale factors normal fp32
    numbers, so a super-block whose largest element is below 2^-97 (about
    6e-30) keeps fewer than 30 bits.  Beside blocks of normal magnitude that is
    far under the row's fp32 resolution; a whole row that small loses accuracy:
    nothing at 1e-29, about 1e-6 at 1e-32, about 1e-3 at 1e-35, and most of
    the value at fp32's smallest normals (1e-38), where the reference's own
    fp32 loop stays near 1e-6.  Activations of a model never sit there."""
    t = synth.IDS[fmt]
    N, K = 128, 4096
    blocks = synth.random_blocks(t, N, K, seed=3)
    W = dequant_f32(t, blocks, N, K).astype(F64)
    base = synth.random_activations(1, K, seed=4)[0].astype(F32)
    for scale, lo, hi in ((1e-29, 0.0, REPR_TOL), (1e-32, 0.0, 3e-6), (1e-35, 1e-4, 3e-3), (1e-38, 0.1, 1.0)):
        x = (base * F32(scale)).astype(F32)
        exact = W @ x.astype(F64)
        err = rel_l2(emulate_kq(t, blocks, x, N, K), exact)
        assert lo <= err <= hi, (scale, err)
        assert rel_l2(np.asarray(oracle_mod.gemv(t, blocks, x, N, K)), exact) <= 1e-5
