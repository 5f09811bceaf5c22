"""The operand roundings of the tcgen05 dequant-GEMM (gemm_tc.cu), restated in
numpy on the CPU, against the oracle restatement of cpu_matmul_transposed_q4_k
/ _q6_k (src/tensor.h:769-856).

The GEMM multiplies fp16 operands with fp32 accumulation:
* weights, dequantized per element in fp16 arithmetic (Dq<T>::emit):
  Q4_K  w = fp16( q * fp16(d sc) + fp16(-dmin m) )   (one fp16 fma)
  Q6_K  w = fp16( (q - 32) * fp16(d sc) )            (one fp16 multiply)
  with d sc and dmin m formed in fp32 (exact) and rounded to fp16 once;
* activations (x_to_f16_kernel): each row scaled by the power of two 2^-k
  that brings its largest magnitude into [2^14, 2^15), rounded to fp16, the
  factor 2^k applied to the row's outputs.

Here the operands get exactly those roundings and the products are summed in
float64, isolating the operand error from the fp32 accumulation: it is
2.5e-4 to 6e-4 relative L2 per output row, which is what the GPU tests bound at
1e-3 (tests/test_gpu_gemm_tc.py) -- three to four orders of magnitude above the
K-quant GEMV forms' representation error (1e-8 to 1e-7, test_gemv_arith.py),
and the reason those forms serve decode."""
import numpy as np
import pytest

from conftest import REL_L2_TOL, rel_l2
from swq import synth
from test_gemv_arith import dequant_f32, q4k_parts, q6k_parts

F16, F32, F64 = np.float16, np.float32, np.float64
Q4_K, Q6_K = synth.IDS["Q4_K"], synth.IDS["Q6_K"]


def tc_weights(t, blocks, N, K) -> np.ndarray:
    """The fp16 weights the GEMM's dequantizer emits, as float64."""
    if t == Q4_K:
        d, dmin, sc, mn, q = q4k_parts(blocks, N, K)
        d1 = (d[..., None] * sc.astype(F32)).astype(F32).astype(F16).astype(F64)     # [N, nb, 8]
        n1 = (-(dmin[..., None] * mn.astype(F32))).astype(F32).astype(F16).astype(F64)
        w = q.astype(F64) * np.repeat(d1, 32, axis=2) + np.repeat(n1, 32, axis=2)  # exact, one rounding
    else:
        d, sc, q = q6k_parts(blocks, N, K)
        ds = (d[..., None] * sc.astype(F32)).astype(F32).astype(F16).astype(F64)     # [N, nb, 16]
        w = q.astype(F64) * np.repeat(ds, 16, axis=2)
    return w.astype(F16).astype(F64).reshape(N, K)


def tc_activations(X: np.ndarray):
    """Rows scaled into [2^14, 2^15), rounded to fp16; the factors back."""
    X = np.asarray(X, F32)
    mx = np.abs(X).max(axis=1).astype(F32)
    k = np.where(mx > 0, np.maximum(((mx.view(np.int32) >> 23) & 0xFF) - 127 - 14, -100), 0)
    xh = (X * np.ldexp(F32(1), -k).astype(F32)[:, None]).astype(F32).astype(F16).astype(F64)
    return xh, np.ldexp(1.0, k)


def emulate_tc(t, blocks, X, N, K) -> np.ndarray:
    xh, back = tc_activations(X)
    return (xh @ tc_weights(t, blocks, N, K).T) * back[:, None]


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("M,N,K", [(9, 256, 4096), (16, 128, 14336)])
def test_tc_operand_error_within_gemm_bound(oracle_mod, fmt, M, N, K):
    t = synth.IDS[fmt]
    blocks = synth.random_blocks(t, N, K, seed=M + N + K)
    X = synth.random_activations(M, K, seed=K - M)
    ref = np.asarray(oracle_mod.gemm(t, blocks, X, M, N, K)).reshape(M, N)
    exact = X.astype(F64) @ dequant_f32(t, blocks, N, K).astype(F64).T
    emu = emulate_tc(t, blocks, X, N, K)
    errs = [rel_l2(emu[m], exact[m]) for m in range(M)]
    assert max(errs) <= REL_L2_TOL, errs
    assert min(errs) >= 1e-5, errs  # fp16 operands: far above the GEMV forms' 1e-7
    for m in range(M):
        assert rel_l2(emu[m], ref[m]) <= REL_L2_TOL


def test_tc_weight_and_activation_parts():
    """Where the error comes from: the weight rounding alone and the
    activation rounding alone, each a few 1e-4 (fp16's 2^-11 unit, averaged
    over the row)."""
    t, N, K, M = Q4_K, 128, 4096, 4
    blocks = synth.random_blocks(t, N, K, seed=21)
    X = synth.random_activations(M, K, seed=22)
    W = dequant_f32(t, blocks, N, K).astype(F64)
    exact = X.astype(F64) @ W.T
    xh, back = tc_activations(X)
    only_w = X.astype(F64) @ tc_weights(t, blocks, N, K).T
    only_x = (xh @ W.T) * back[:, None]
    for m in range(M):
        for got in (only_w, only_x):
            assert 1e-5 <= rel_l2(got[m], exact[m]) <= 1e-3
