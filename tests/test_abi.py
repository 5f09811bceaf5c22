"""The C ABI of libswq on the CPU: the library loads, exports every function
include/swq.h declares, and rejects bad arguments with the documented status
before touching a GPU (no compute call runs here)."""
import ctypes

import pytest

import kat
import swq
from swq.lib import Status, lib


def test_library_built_and_loads():
    assert swq.lib_path().exists(), "run __graft_entry__.build() first"
    lib()


def test_exports_every_header_symbol():
    declared = swq.header_symbols()
    assert {"swq_dequant", "swq_gemv", "swq_gemm", "swq_ctx_matmul_transposed_q"} <= set(declared)
    exported = set(swq.exported_symbols())
    missing = [s for s in declared if s not in exported]
    assert not missing, f"declared in include/swq.h but not exported: {missing}"
    for s in declared:
        getattr(lib(), s)


def test_type_and_block_sizes():
    for t, bb in kat.TYPE_SIZES.items():
        assert swq.type_size(t) == bb
        assert swq.block_size(t) == kat.BLOCK_SIZES[t]
    for t in (0, 1, 6, 30, 37):  # F32, F16, Q5_0, BF16, F8 are not on this path
        assert swq.type_size(t) == 0 and swq.block_size(t) == 0


def test_status_strings():
    L = lib()
    for s in Status:
        assert L.swq_status_string(int(s))


def _rc(fn, *args):
    return Status(fn(*args))


def test_gemv_argument_errors():
    L = lib()
    assert _rc(L.swq_gemv, 0, 1, 1, 1, 4, 256, None) is Status.BAD_TYPE
    assert _rc(L.swq_gemv, kat.Q4_K, 1, 1, 1, 4, 100, None) is Status.BAD_SHAPE
    assert b"multiple of 256" in L.swq_last_error()
    assert _rc(L.swq_gemv, kat.Q4_0, 1, 1, 1, 4, 48, None) is Status.BAD_SHAPE
    assert _rc(L.swq_gemv, kat.Q4_K, None, 1, 1, 4, 256, None) is Status.NULL_PTR
    assert _rc(L.swq_gemv, kat.Q4_K, 1, None, 1, 4, 256, None) is Status.NULL_PTR
    assert _rc(L.swq_gemv, kat.Q4_K, 1, 1, None, 4, 256, None) is Status.NULL_PTR
    assert _rc(L.swq_gemm, kat.Q4_K, 1, 1, 1, -1, 4, 256, None) is Status.BAD_SHAPE
    # empty problems are a no-op, like the reference's loops over zero rows
    assert _rc(L.swq_gemv, kat.Q4_K, None, None, None, 0, 256, None) is Status.OK
    assert _rc(L.swq_gemm, kat.Q4_K, None, None, None, 0, 4, 256, None) is Status.OK


def test_prefill_argument_errors():
    """Prompt rows past the cache, unsupported head sizes, null pointers: each
    rejected before anything runs; zero rows is a no-op."""
    L = lib()
    # rope: (q, k, v, kc, vc, pos0, seq_len, freqs, q_dim, kv_dim, head_dim, rope_dim, neox, seqs, max_seq, ld x3)
    rope = lambda pos0, P, hd=64, rd=64, seqs=1, q=1: _rc(  # noqa: E731
        L.swq_rope_kv_prefill, q, 1, 1, 1, 1, pos0, P, 1, 512, 128, hd, rd, 0, seqs, 16, 0, 0, 0, None)
    assert rope(10, 7) is Status.BAD_SHAPE           # positions 10..16 past max_seq 16
    assert b"max_seq" in L.swq_last_error()
    assert rope(-1, 2) is Status.BAD_SHAPE
    assert rope(0, 4, rd=63) is Status.BAD_SHAPE     # odd rotary dimension
    assert rope(0, 4, hd=96) is Status.BAD_SHAPE     # 512 is not a multiple of 96
    assert rope(0, 4, q=None) is Status.NULL_PTR
    assert rope(0, 0, q=None) is Status.OK           # no rows
    assert rope(0, 4, seqs=0, q=None) is Status.OK
    # attention: (out, q, kc, vc, pos0, seq_len, heads, kv_heads, head_dim, seqs, max_seq, ldq, ldo)
    att = lambda pos0, P, H=8, Hkv=2, hd=64, out=1, ldq=0: _rc(  # noqa: E731
        L.swq_attention_prefill, out, 1, 1, 1, pos0, P, H, Hkv, hd, 1, 16, ldq, 0, None)
    assert att(0, 17) is Status.BAD_SHAPE
    assert att(0, 4, Hkv=3) is Status.BAD_SHAPE      # kv heads must divide query heads
    assert att(0, 4, hd=96) is Status.BAD_SHAPE      # head_dim 32/64/128/256
    assert att(0, 4, ldq=100) is Status.BAD_SHAPE    # row stride below 8 x 64
    assert att(0, 4, out=None) is Status.NULL_PTR
    assert att(0, 0, out=None) is Status.OK


def test_qkv_bias_norm_argument_errors():
    L = lib()
    # (q, k, v, bq, bk, bv, q_norm, k_norm, q_dim, kv_dim, head_dim, eps, rows, ldq, ldk, ldv)
    def f(q=1, k=1, v=1, bq=1, bk=None, bv=None, qn=None, kn=None, hd=64, rows=2, ldq=0):
        return _rc(L.swq_qkv_bias_norm, q, k, v, bq, bk, bv, qn, kn, 512, 128, hd, 1e-5, rows, ldq, 0, 0, None)

    assert f(hd=96) is Status.BAD_SHAPE            # 512 is not a multiple of 96
    assert f(ldq=100) is Status.BAD_SHAPE          # row stride below q_dim
    assert f(rows=-1) is Status.BAD_SHAPE
    assert f(q=None) is Status.NULL_PTR            # a q bias with no q
    assert f(k=None, kn=1, bq=None) is Status.NULL_PTR
    assert f(q=None, k=None, v=None, bq=None) is Status.OK   # no bias, no norm: nothing to do
    assert f(rows=0, q=None) is Status.OK


def test_dequant_argument_errors():
    L = lib()
    assert _rc(L.swq_dequant, 1, 1, 1, 32, None) is Status.BAD_TYPE
    assert _rc(L.swq_dequant, kat.Q8_0, 1, 1, -32, None) is Status.BAD_SHAPE
    assert _rc(L.swq_dequant, kat.Q8_0, None, 1, 32, None) is Status.NULL_PTR
    # fewer elements than one block: nothing to write (reference: n / QK blocks)
    assert _rc(L.swq_dequant, kat.Q4_K, None, None, 255, None) is Status.OK
    assert _rc(L.swq_dequant, kat.Q4_K, None, None, 0, None) is Status.OK


def test_options():
    assert swq.get_option(swq.OPT_Q2K_REFERENCE_CPU_ORDER) == 1
    assert swq.get_option(swq.OPT_EARLY_WEIGHT_PREFETCH) == 1
    assert swq.get_option(swq.OPT_TENSOR_CORE_GEMM) == 1
    swq.set_option(swq.OPT_TENSOR_CORE_GEMM, 0)
    assert swq.get_option(swq.OPT_TENSOR_CORE_GEMM) == 0
    swq.set_option(swq.OPT_TENSOR_CORE_GEMM, 1)
    with pytest.raises(swq.SwqError):
        swq.set_option(swq.OPT_TENSOR_CORE_GEMM, 2)
    assert swq.get_option(swq.OPT_TENSOR_CORE_MIN_M) == 5
    with pytest.raises(swq.SwqError):
        swq.set_option(swq.OPT_TENSOR_CORE_MIN_M, 1)
    swq.set_option(swq.OPT_Q2K_REFERENCE_CPU_ORDER, 0)
    assert swq.get_option(swq.OPT_Q2K_REFERENCE_CPU_ORDER) == 0
    swq.set_option(swq.OPT_Q2K_REFERENCE_CPU_ORDER, 1)
    assert swq.get_option(swq.OPT_GEMV_FP32_ACT) == 1
    assert swq.get_option(swq.OPT_GEMV_INT_MMA) == 2
    for opt, bad in ((swq.OPT_GEMV_FP32_ACT, 2), (swq.OPT_GEMV_INT_MMA, 3), (swq.OPT_GEMV_INT_MMA, -1)):
        with pytest.raises(swq.SwqError):
            swq.set_option(opt, bad)
    with pytest.raises(swq.SwqError) as ei:
        swq.set_option(swq.OPT_GEMV_MAX_M, 9)
    assert ei.value.status is Status.BAD_ARG
    # batched K-quant GEMV: up to 16 rows; table size and tile groups automatic
    assert swq.get_option(swq.OPT_GEMV_BATCH_MAX_M) == 16
    assert swq.get_option(swq.OPT_GEMV_BATCH_TABLE_KB) == 0
    assert swq.get_option(swq.OPT_GEMV_BATCH_GROUP) == 0
    swq.set_option(swq.OPT_GEMV_BATCH_TABLE_KB, 144)
    assert swq.get_option(swq.OPT_GEMV_BATCH_TABLE_KB) == 144
    swq.set_option(swq.OPT_GEMV_BATCH_TABLE_KB, 0)
    for opt, bad in ((swq.OPT_GEMV_BATCH_TABLE_KB, 7), (swq.OPT_GEMV_BATCH_TABLE_KB, 161),
                     (swq.OPT_GEMV_BATCH_GROUP, 3), (swq.OPT_GEMV_BATCH_GROUP, 32)):
        with pytest.raises(swq.SwqError):
            swq.set_option(opt, bad)
    with pytest.raises(swq.SwqError):
        swq.set_option(99, 0)
    assert swq.get_option(99) == -1


def test_ctx_null_handle_errors():
    L = lib()
    assert _rc(L.swq_ctx_matmul_transposed_q, None, 1, 1, 1, kat.Q4_K, 4, 256) is Status.NULL_PTR
    assert _rc(L.swq_ctx_create, 0, None) is Status.NULL_PTR
    assert _rc(L.swq_ctx_destroy, None) is Status.OK
    assert L.swq_ctx_resident_bytes(None) == 0
    out = ctypes.c_void_p()
    assert isinstance(out, ctypes.c_void_p)


def test_grouped_gemm_argument_checks():
    """swq_grouped_gemm rejects bad arguments before any device work."""
    L = swq.lib()
    assert _rc(L.swq_grouped_gemm, 99, 16, 16, 16, 16, 4, 8, 64, 256, None) is Status.BAD_TYPE
    assert _rc(L.swq_grouped_gemm, kat.Q4_K, 16, 16, 16, 16, 4, 8, 64, 100, None) is Status.BAD_SHAPE
    assert _rc(L.swq_grouped_gemm, kat.Q4_K, 16, 16, 16, 16, 5000, 8, 64, 256, None) is Status.BAD_SHAPE
    assert _rc(L.swq_grouped_gemm, kat.Q4_K, None, 16, 16, 16, 4, 8, 64, 256, None) is Status.NULL_PTR
    # nothing to do: no rows
    assert _rc(L.swq_grouped_gemm, kat.Q4_K, None, None, None, None, 4, 0, 64, 256, None) is Status.OK
