"""The oracle (oracle/swq_oracle.c) pinned against the reference.

1. the known-answer blocks of the reference's tests/test_gguf.cpp;
2. golden vectors produced by the reference's own src/tensor.h compiled from
   source (tests/golden/make_golden.py), bit-exact;
3. where oracle/_ref was built (the reference tree is mounted), the compiled
   reference itself on fresh seeded inputs, bit-exact.
"""
import numpy as np
import pytest

import kat
from conftest import rel_l2
from swq import synth

FORMATS = ["Q4_0", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]


def test_type_and_block_sizes(oracle_mod):
    lib = oracle_mod.oracle_lib()
    for t, bb in kat.TYPE_SIZES.items():
        assert lib.oracle_type_size(t) == bb
        assert lib.oracle_block_size(t) == kat.BLOCK_SIZES[t]
    assert lib.oracle_type_size(0) == 0  # F32 is not on this path


def test_fp16_conversion(oracle_mod):
    for h, v in kat.FP16_CASES:
        assert oracle_mod.fp16_to_fp32(h) == v


def test_fp16_conversion_all_halves_match_numpy(oracle_mod):
    # Every finite half (incl. subnormals) converts exactly; Inf keeps sign.
    for h in list(range(0, 0x7C01, 97)) + [0x0001, 0x03FF, 0x0400, 0x7BFF, 0x7C00, 0xFC00, 0x8001]:
        ref = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        assert oracle_mod.fp16_to_fp32(h) == ref


@pytest.mark.parametrize("case", kat.dequant_kats(), ids=lambda c: c["name"])
def test_dequant_known_answers(oracle_mod, case):
    out = oracle_mod.dequantize(case["type"], case["blocks"], case["n"])
    np.testing.assert_allclose(out[case["sl"]], case["value"], atol=case["tol"])


def test_fused_q8_0_known_answer(oracle_mod):
    c = kat.q8_0_2x32()
    out = oracle_mod.gemv(c["type"], c["blocks"], c["x"], c["N"], c["K"])
    np.testing.assert_allclose(out, c["expect"], atol=c["tol"])
    dq = oracle_mod.dequantize(c["type"], c["blocks"], c["N"] * c["K"])
    np.testing.assert_allclose(out, dq.reshape(2, 32) @ c["x"], atol=1e-4)


def test_fused_q4_0_known_answer(oracle_mod):
    c = kat.q4_0_2x32()
    dq = oracle_mod.dequantize(c["type"], c["blocks"], 64).reshape(2, 32)
    for x in (c["x"], c["x_alt"]):
        out = oracle_mod.gemv(c["type"], c["blocks"], x, 2, 32)
        np.testing.assert_allclose(out, dq @ x, atol=1e-4)
    out = oracle_mod.gemv(c["type"], c["blocks"], c["x"], 2, 32)
    np.testing.assert_allclose(out, c["expect"], atol=c["tol"])


@pytest.mark.parametrize("case", kat.fused_kats(), ids=lambda c: c["name"])
def test_fused_kquant_known_answers(oracle_mod, case):
    x = np.ones(case["K"], np.float32)
    out = oracle_mod.gemv(case["type"], case["blocks"], x, case["N"], case["K"])
    dq = oracle_mod.dequantize(case["type"], case["blocks"], case["N"] * case["K"]).reshape(case["N"], case["K"])
    np.testing.assert_allclose(out, dq @ x, atol=case["tol"])
    if case["expect"] is not None:
        np.testing.assert_allclose(out, case["expect"], atol=case["tol"])


@pytest.mark.parametrize("fmt", FORMATS)
def test_oracle_matches_reference_golden(oracle_mod, golden, fmt):
    g = golden(fmt)
    t, N, K = int(g["type"]), int(g["N"]), int(g["K"])
    dq = oracle_mod.dequantize(t, g["blocks"], N * K)
    assert np.array_equal(dq.view(np.uint32), g["dequant"].view(np.uint32))
    for m in range(g["x"].shape[0]):
        ref_order = oracle_mod.gemv(t, g["blocks"], g["x"][m], N, K, format_order=False)
        assert np.array_equal(ref_order.view(np.uint32), g["gemv_ref"][m].view(np.uint32))
        fmt_order = oracle_mod.gemv(t, g["blocks"], g["x"][m], N, K, format_order=True)
        if fmt == "Q2_K":
            # dequantize_q2_k order == reference dequantize + fp32 GEMV, bit-exact
            assert np.array_equal(fmt_order.view(np.uint32), g["gemv_dq"][m].view(np.uint32))
        else:
            assert np.array_equal(fmt_order.view(np.uint32), ref_order.view(np.uint32))
            assert rel_l2(fmt_order, g["gemv_dq"][m]) < 1e-5


def test_reference_q2k_fused_differs_from_its_dequantizer(golden):
    """Pins the discrepancy inside the reference: cpu_matmul_transposed_q2_k
    (src/tensor.h:935-945) does not equal dequantize_q2_k + dot."""
    g = golden("Q2_K")
    assert rel_l2(g["gemv_ref"], g["gemv_dq"]) > 0.5


def test_special_scales_golden(oracle_mod, golden):
    g = dict(np.load(__import__("conftest").GOLDEN / "golden_special_scales.npz"))
    for name in ("Q4_K", "Q6_K", "Q8_0"):
        t = synth.IDS[name]
        blocks = g[f"{name}_blocks"]
        n = blocks.size // synth.block_geometry(t)[1] * synth.block_geometry(t)[0]
        out = oracle_mod.dequantize(t, blocks, n)
        assert np.array_equal(out.view(np.uint32), g[f"{name}_dequant"].view(np.uint32))


@pytest.mark.parametrize("fmt", FORMATS)
def test_oracle_matches_compiled_reference(oracle_mod, fmt):
    if not oracle_mod.ref_available():
        pytest.skip("oracle/_ref not built here (reference sources absent)")
    t = synth.IDS[fmt]
    N, K = 33, 2048
    blocks = synth.random_blocks(t, N, K, seed=77 + t)
    x = synth.random_activations(1, K, seed=78)[0]
    a = oracle_mod.dequantize(t, blocks, N * K)
    b = oracle_mod.ref_dequantize(t, blocks, N * K)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    ga = oracle_mod.gemv(t, blocks, x, N, K, format_order=False)
    gb = oracle_mod.ref_gemv(t, blocks, x, N, K)
    assert np.array_equal(ga.view(np.uint32), gb.view(np.uint32))


def test_oracle_batched_equals_rowwise(oracle_mod):
    t = synth.Q4_K
    N, K, M = 8, 512, 3
    blocks = synth.random_blocks(t, N, K, seed=5)
    X = synth.random_activations(M, K, seed=6)
    Y = oracle_mod.gemm(t, blocks, X, M, N, K)
    for m in range(M):
        assert np.array_equal(Y[m], oracle_mod.gemv(t, blocks, X[m], N, K))


def test_oracle_rejects_unknown_type(oracle_mod):
    with pytest.raises(ValueError):
        oracle_mod.dequantize(0, np.zeros(4, np.uint8), 1)
