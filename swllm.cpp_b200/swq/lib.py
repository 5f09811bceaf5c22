"""ctypes binding of libswq.so (include/swq.h)."""
from __future__ import annotations

import ctypes
import enum
import re
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG_ROOT = HERE.parent                      # swllm.cpp_b200/
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
HEADER = REPO_ROOT / "include" / "swq.h"
_LIB_PATH = HERE / "libswq.so"

# GGMLType ids, src/gguf.h:18-40
Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 2, 8, 10, 11, 12, 13, 14
TYPES = {"Q4_0": Q4_0, "Q8_0": Q8_0, "Q2_K": Q2_K, "Q3_K": Q3_K,
         "Q4_K": Q4_K, "Q5_K": Q5_K, "Q6_K": Q6_K}
TYPE_NAMES = {v: k for k, v in TYPES.items()}

OPT_Q2K_REFERENCE_CPU_ORDER = 1
OPT_EARLY_WEIGHT_PREFETCH = 2
OPT_GEMV_MAX_M = 3
OPT_TENSOR_CORE_GEMM = 4
OPT_TENSOR_CORE_MIN_M = 5
OPT_GEMV_SMEM_KB = 6
OPT_GEMV_STAGE_KB = 7
OPT_GEMV_CTAS_PER_SM = 8
OPT_GEMV_FP32_ACT = 9
OPT_GEMV_INT_MMA = 10
OPT_GEMV_BATCH_MAX_M = 11
OPT_GEMV_BATCH_TABLE_KB = 12
OPT_GEMV_BATCH_GROUP = 13
OPT_PREFILL_ATTENTION = 14

GEMM_NOALLOC_MAX_X_ELEMS = 8388608  # SWQ_GEMM_NOALLOC_MAX_X_ELEMS


class Status(enum.IntEnum):
    OK = 0
    BAD_TYPE = 1
    BAD_SHAPE = 2
    NULL_PTR = 3
    CUDA = 4
    TIMEOUT = 5
    UNSUPPORTED = 6
    BAD_ARG = 7


class SwqError(RuntimeError):
    def __init__(self, status: int, detail: str):
        self.status = Status(status)
        super().__init__(f"swq: {self.status.name}: {detail}")


_lib = None


def lib_path() -> Path:
    return _LIB_PATH


def build(jobs: int = 8) -> Path:
    """Compile libswq.so for sm_100a (nvcc cross-compiles without a GPU)."""
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", str(CSRC)], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        raise FileNotFoundError(f"{_LIB_PATH} is not built; run swq.build() (make -C {CSRC})")
    L = ctypes.CDLL(str(_LIB_PATH))
    vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
    sig = {
        "swq_status_string": (ctypes.c_char_p, [i32]),
        "swq_last_error": (ctypes.c_char_p, []),
        "swq_type_size": (sz, [i32]),
        "swq_block_size": (sz, [i32]),
        "swq_dequant": (i32, [i32, vp, vp, i64, vp]),
        "swq_gemv": (i32, [i32, vp, vp, vp, i32, i32, vp]),
        "swq_gemm": (i32, [i32, vp, vp, vp, i32, i32, i32, vp]),
        "swq_gemm_noalloc": (i32, [i32, vp, vp, vp, i32, i32, i32, vp]),
        "swq_gemm_act": (i32, [i32, vp, vp, vp, i32, i32, i32, ctypes.POINTER(ActArgs), i32, vp]),
        "swq_gemm_workspace_bytes": (sz, [i32, i32, i32, i32]),
        "swq_gemm_act_ws": (i32, [i32, vp, vp, vp, i32, i32, i32, ctypes.POINTER(ActArgs), vp, sz, vp]),
        "swq_grouped_gemm": (i32, [i32, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
        "swq_grouped_gemv": (i32, [i32, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
        "swq_grouped_matmul": (i32, [i32, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
        "swq_grouped_matmul_stacked": (i32, [i32, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
        "swq_moe_router": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp]),
        "swq_moe_sort": (i32, [vp, i32, i32, vp, vp, vp, vp]),
        "swq_moe_gather": (i32, [vp, vp, vp, i32, i32, i32, i32, vp, vp]),
        "swq_moe_combine": (i32, [vp, vp, vp, i32, i32, i32, vp, i32, vp]),
        "swq_ep_create": (i32, [i32, i32, i32, i32, i32, i32, ctypes.POINTER(vp), vp]),
        "swq_ep_open": (i32, [vp, vp]),
        "swq_ep_dispatch": (i32, [vp, vp, vp, i32, vp]),
        "swq_ep_received": (i32, [vp, ctypes.POINTER(vp), ctypes.POINTER(vp), ctypes.POINTER(i32)]),
        "swq_ep_combine": (i32, [vp, vp, vp, vp, i32, vp]),
        "swq_ep_reset": (i32, [vp, vp]),
        "swq_ep_destroy": (i32, [vp]),
        "swq_rmsnorm": (i32, [vp, vp, vp, i32, ctypes.c_float, i32, vp]),
        "swq_add_rmsnorm": (i32, [vp, vp, vp, vp, i32, ctypes.c_float, i32, vp]),
        "swq_rope_kv": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32, vp]),
        "swq_attention_workspace_bytes": (sz, [i32, i32, i32, i32, i32]),
        "swq_attention_decode": (i32, [vp, vp, vp, vp, vp, vp, sz, i32, i32, i32, i32, i32, i32, vp]),
        "swq_rope_kv_prefill": (i32, [vp, vp, vp, vp, vp, i32, i32, vp, i32, i32, i32, i32, i32, i32, i32, i32,
                                      i32, i32, vp]),
        "swq_attention_prefill": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, i32, i32, vp]),
        "swq_qkv_bias_norm": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, ctypes.c_float, i32, i32, i32,
                                    i32, vp]),
        "swq_gdn_step": (i32, [vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]),
        "swq_silu_mul": (i32, [vp, vp, vp, i32, i32, i32, vp]),
        "swq_add": (i32, [vp, vp, i64, vp]),
        "swq_embed": (i32, [vp, vp, vp, i32, i32, i32, vp]),
        "swq_argmax": (i32, [vp, i32, i32, vp, vp, vp, vp]),
        "swq_decode_advance": (i32, [vp, vp, vp]),
        "swq_set_option": (i32, [i32, i32]),
        "swq_get_option": (i32, [i32]),
        "swq_check": (i32, [vp]),
        "swq_allreduce_create": (i32, [sz, i32, i32, ctypes.POINTER(vp), vp]),
        "swq_allreduce_open": (i32, [vp, vp]),
        "swq_allreduce_sum": (i32, [vp, vp, sz, vp]),
        "swq_allreduce_reset": (i32, [vp, vp]),
        "swq_allreduce_destroy": (i32, [vp]),
        "swq_ctx_create": (i32, [i32, ctypes.POINTER(vp)]),
        "swq_ctx_destroy": (i32, [vp]),
        "swq_ctx_matmul_transposed_q": (i32, [vp, vp, vp, vp, i32, i32, i32]),
        "swq_ctx_matmul_q_batched": (i32, [vp, vp, vp, vp, i32, i32, i32, i32]),
        "swq_ctx_dequantize": (i32, [vp, vp, vp, i64, i32]),
        "swq_ctx_evict": (i32, [vp, vp]),
        "swq_ctx_resident_bytes": (sz, [vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _raise(rc: int) -> None:
    if rc != 0:
        detail = lib().swq_last_error().decode(errors="replace")
        raise SwqError(rc, detail)


def header_symbols() -> list[str]:
    """Every function declared in include/swq.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*[\w\s\*]+?\b(swq_\w+)\s*\(", text, flags=re.M)))


def exported_symbols() -> list[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(_LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    return sorted({ln.split()[-1] for ln in out.splitlines() if ln.split() and ln.split()[-1].startswith("swq_")})


def type_size(t: int) -> int:
    return int(lib().swq_type_size(t))


def block_size(t: int) -> int:
    return int(lib().swq_block_size(t))


def set_option(opt: int, value: int) -> None:
    _raise(lib().swq_set_option(opt, value))


def get_option(opt: int) -> int:
    return int(lib().swq_get_option(opt))


def _ptr(a) -> int:
    """Device address of a torch tensor, or an int address as given."""
    if a is None:
        return 0
    if isinstance(a, int):
        return a
    return int(a.data_ptr())


def _stream(stream) -> int:
    if stream is None:
        try:
            import torch
            if torch.cuda.is_available():
                return int(torch.cuda.current_stream().cuda_stream)
        except Exception:  # pragma: no cover
            pass
        return 0
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


def dequant(type_id: int, blocks, out, n: int, stream=None) -> None:
    """out[:n] = dequantize(blocks) on the device, bit-exact (async)."""
    _raise(lib().swq_dequant(type_id, _ptr(blocks), _ptr(out), n, _stream(stream)))


def gemv(type_id: int, W, x, y, N: int, K: int, stream=None) -> None:
    """y[N] = W[N x K] . x[K] on device buffers (async)."""
    _raise(lib().swq_gemv(type_id, _ptr(W), _ptr(x), _ptr(y), N, K, _stream(stream)))


def gemm(type_id: int, W, X, Y, M: int, N: int, K: int, stream=None) -> None:
    """Y[M x N] = X[M x K] . W[N x K]^T on device buffers (async)."""
    _raise(lib().swq_gemm(type_id, _ptr(W), _ptr(X), _ptr(Y), M, N, K, _stream(stream)))


def grouped_gemm(type_id: int, w_ptrs, offsets, X, Y, n_experts: int, total_rows: int, N: int, K: int,
                 stream=None) -> None:
    """MoE grouped GEMM: rows offsets[e] .. offsets[e+1]-1 of X times W_e^T into
    the same rows of Y.  w_ptrs: device int64 tensor of the experts' weight
    addresses; offsets: device int32 tensor of n_experts + 1 row offsets."""
    _raise(lib().swq_grouped_gemm(type_id, _ptr(w_ptrs), _ptr(offsets), _ptr(X), _ptr(Y), n_experts, total_rows,
                                  N, K, _stream(stream)))


def grouped_matmul(type_id: int, w_ptrs, offsets, X, Y, n_experts: int, total_rows: int, N: int, K: int,
                   mean_rows: int, stream=None) -> None:
    """Grouped expert product with the kernel picked from mean_rows, the
    expected rows per expert (swq_grouped_matmul); total_rows bounds the rows."""
    _raise(lib().swq_grouped_matmul(type_id, _ptr(w_ptrs), _ptr(offsets), _ptr(X), _ptr(Y), n_experts, total_rows,
                                    N, K, mean_rows, _stream(stream)))


def grouped_matmul_stacked(type_id: int, W_all, offsets, X, Y, n_experts: int, total_rows: int, N: int, K: int,
                           mean_rows: int, stream=None) -> None:
    """grouped_matmul with expert e at rows e*N .. of one stacked tensor W_all."""
    _raise(lib().swq_grouped_matmul_stacked(type_id, _ptr(W_all), _ptr(offsets), _ptr(X), _ptr(Y), n_experts,
                                            total_rows, N, K, mean_rows, _stream(stream)))


def moe_router(router_w, X, T: int, E: int, H: int, k: int, logits, ids, w, stream=None) -> None:
    """fp32 router GEMV into logits [T, E], top-k ids [T, k] (int32) and the
    softmax over those k logits w [T, k] (swq_moe_router)."""
    _raise(lib().swq_moe_router(_ptr(router_w), _ptr(X), T, E, H, k, _ptr(logits), _ptr(ids), _ptr(w),
                                _stream(stream)))


def moe_sort(ids, P: int, n_experts: int, offsets, sorted_pairs, pair_rows, stream=None) -> None:
    """Stable sort of P (token, slot) pairs by expert (swq_moe_sort)."""
    _raise(lib().swq_moe_sort(_ptr(ids), P, n_experts, _ptr(offsets), _ptr(sorted_pairs), _ptr(pair_rows),
                              _stream(stream)))


def moe_gather(X, sorted_pairs, offsets, n_experts: int, P: int, k: int, H: int, X_sorted, stream=None) -> None:
    """X_sorted[r] = X[sorted_pairs[r] // k] for the sorted rows (swq_moe_gather)."""
    _raise(lib().swq_moe_gather(_ptr(X), _ptr(sorted_pairs), _ptr(offsets), n_experts, P, k, H, _ptr(X_sorted),
                                _stream(stream)))


def moe_combine(Y_sorted, pair_rows, w, T: int, k: int, H: int, Y, accumulate: bool = False, stream=None) -> None:
    """Y[t] (+)= sum_j w[t, j] * Y_sorted[pair_rows[t*k + j]] (swq_moe_combine)."""
    _raise(lib().swq_moe_combine(_ptr(Y_sorted), _ptr(pair_rows), _ptr(w), T, k, H, _ptr(Y), 1 if accumulate else 0,
                                 _stream(stream)))


ACT_NONE, ACT_RMSNORM, ACT_SWIGLU = 0, 1, 2
GEMM_NOALLOC = 1


class ActArgs(ctypes.Structure):
    """swq_act (include/swq.h)."""
    _fields_ = [("kind", ctypes.c_int), ("residual", ctypes.c_void_p), ("norm_w", ctypes.c_void_p),
                ("eps", ctypes.c_float), ("sum_out", ctypes.c_void_p), ("ld", ctypes.c_int)]


def gemm_act(type_id: int, W, X, Y, M: int, N: int, K: int, kind: int = ACT_NONE, residual=None, norm_w=None,
             eps: float = 0.0, sum_out=None, ld: int = 0, noalloc: bool = False, stream=None) -> None:
    """gemm() on a transformed X (swq_gemm_act): RMSNORM of X (+ residual),
    weights norm_w, the sum written to sum_out; or SWIGLU of the gate/up row
    halves (row stride ld, 0 = 2K)."""
    a = ActArgs(kind, _ptr(residual) if residual is not None else None,
                _ptr(norm_w) if norm_w is not None else None, eps,
                _ptr(sum_out) if sum_out is not None else None, ld)
    _raise(lib().swq_gemm_act(type_id, _ptr(W), _ptr(X), _ptr(Y), M, N, K, ctypes.byref(a),
                              GEMM_NOALLOC if noalloc else 0, _stream(stream)))


def gemm_workspace_bytes(type_id: int, M: int, N: int, K: int) -> int:
    """Workspace bytes gemm_act_ws needs for this shape on the current device
    (0 when the GEMV kernel serves it)."""
    return int(lib().swq_gemm_workspace_bytes(type_id, M, N, K))


def gemm_act_ws(type_id: int, W, X, Y, M: int, N: int, K: int, workspace, workspace_bytes: int,
                kind: int = ACT_NONE, residual=None, norm_w=None, eps: float = 0.0, sum_out=None, ld: int = 0,
                stream=None) -> None:
    """gemm_act() with the tensor-core path's scratch in `workspace` (a device
    buffer of at least gemm_workspace_bytes(), 256-byte aligned, owned by the
    caller): nothing is allocated, and callers with separate workspaces never
    share scratch."""
    a = ActArgs(kind, _ptr(residual) if residual is not None else None,
                _ptr(norm_w) if norm_w is not None else None, eps,
                _ptr(sum_out) if sum_out is not None else None, ld)
    _raise(lib().swq_gemm_act_ws(type_id, _ptr(W), _ptr(X), _ptr(Y), M, N, K, ctypes.byref(a),
                                 _ptr(workspace) if workspace is not None else None, workspace_bytes,
                                 _stream(stream)))


def grouped_gemv(type_id: int, w_ptrs, offsets, X, Y, n_experts: int, total_rows: int, N: int, K: int,
                 stream=None) -> None:
    """grouped_gemm for a few rows per expert (MoE decode): a GEMV per expert's
    rows; every expert matrix must be 16-byte aligned."""
    _raise(lib().swq_grouped_gemv(type_id, _ptr(w_ptrs), _ptr(offsets), _ptr(X), _ptr(Y), n_experts, total_rows,
                                  N, K, _stream(stream)))


def gemm_noalloc(type_id: int, W, X, Y, M: int, N: int, K: int, stream=None) -> None:
    """gemm() without any device allocation: the fp16 copy of X lives in
    libswq's fixed per-device array (M * K <= GEMM_NOALLOC_MAX_X_ELEMS).
    Calls that overlap on the GPU share that array and race."""
    _raise(lib().swq_gemm_noalloc(type_id, _ptr(W), _ptr(X), _ptr(Y), M, N, K, _stream(stream)))


# ---- decode step (device pointers or torch tensors; async on `stream`) ----
def rmsnorm(out, x, w, n: int, eps: float, rows: int = 1, stream=None) -> None:
    _raise(lib().swq_rmsnorm(_ptr(out), _ptr(x), _ptr(w), n, eps, rows, _stream(stream)))


def add_rmsnorm(out, x, y, w, n: int, eps: float, rows: int = 1, stream=None) -> None:
    _raise(lib().swq_add_rmsnorm(_ptr(out), _ptr(x), _ptr(y), _ptr(w), n, eps, rows, _stream(stream)))


def rope_kv(q, k, v, k_cache, v_cache, pos, freqs, q_dim: int, kv_dim: int, head_dim: int, rope_dim: int,
            neox: bool, rows: int, max_seq: int, ldq: int = 0, ldk: int = 0, ldv: int = 0, stream=None) -> None:
    _raise(lib().swq_rope_kv(_ptr(q), _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), _ptr(pos), _ptr(freqs), q_dim,
                             kv_dim, head_dim, rope_dim, 1 if neox else 0, rows, max_seq, ldq, ldk, ldv,
                             _stream(stream)))


def attention_workspace_bytes(num_heads: int, num_kv_heads: int, head_dim: int, rows: int, max_seq: int) -> int:
    return int(lib().swq_attention_workspace_bytes(num_heads, num_kv_heads, head_dim, rows, max_seq))


def attention_decode(out, q, k_cache, v_cache, pos, workspace, workspace_bytes: int, num_heads: int,
                     num_kv_heads: int, head_dim: int, rows: int, max_seq: int, ldq: int = 0, stream=None) -> None:
    _raise(lib().swq_attention_decode(_ptr(out), _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(pos), _ptr(workspace),
                                      workspace_bytes, num_heads, num_kv_heads, head_dim, rows, max_seq, ldq,
                                      _stream(stream)))


def rope_kv_prefill(q, k, v, k_cache, v_cache, pos0: int, seq_len: int, freqs, q_dim: int, kv_dim: int,
                    head_dim: int, rope_dim: int, neox: bool, num_seqs: int, max_seq: int, ldq: int = 0, ldk: int = 0,
                    ldv: int = 0, stream=None) -> None:
    """RoPE + KV append for prompt rows m = s*seq_len + p at position pos0 + p."""
    _raise(lib().swq_rope_kv_prefill(_ptr(q), _ptr(k), _ptr(v), _ptr(k_cache), _ptr(v_cache), pos0, seq_len,
                                     _ptr(freqs), q_dim, kv_dim, head_dim, rope_dim, 1 if neox else 0, num_seqs,
                                     max_seq, ldq, ldk, ldv, _stream(stream)))


def attention_prefill(out, q, k_cache, v_cache, pos0: int, seq_len: int, num_heads: int, num_kv_heads: int,
                      head_dim: int, num_seqs: int, max_seq: int, ldq: int = 0, ldo: int = 0, stream=None) -> None:
    """Causal attention of prompt rows m = s*seq_len + p over positions 0 .. pos0 + p."""
    _raise(lib().swq_attention_prefill(_ptr(out), _ptr(q), _ptr(k_cache), _ptr(v_cache), pos0, seq_len, num_heads,
                                       num_kv_heads, head_dim, num_seqs, max_seq, ldq, ldo, _stream(stream)))


def qkv_bias_norm(q, k, v, bq, bk, bv, q_norm, k_norm, q_dim: int, kv_dim: int, head_dim: int, eps: float,
                  rows: int, ldq: int = 0, ldk: int = 0, ldv: int = 0, stream=None) -> None:
    """q/k/v bias adds, then per-head RMSNorm of q and k (any vector may be None)."""
    _raise(lib().swq_qkv_bias_norm(_ptr(q), _ptr(k), _ptr(v), _ptr(bq), _ptr(bk), _ptr(bv), _ptr(q_norm),
                                   _ptr(k_norm), q_dim, kv_dim, head_dim, eps, rows, ldq, ldk, ldv, _stream(stream)))


def gdn_step(qkv, z, beta, alpha, dt, ssm_a, conv_w, norm_w, state, conv_state, y, rows: int, n_k_heads: int,
             n_v_heads: int, key_head_dim: int, value_head_dim: int, conv_width: int, ld_qkv: int = 0,
             stream=None) -> None:
    """One GatedDeltaNet decode step after the projections (swq_gdn_step):
    conv1d of v, the gated delta-rule update of `state` and its read-out,
    per-head RMSNorm, sigmoid(z) gate, into y.  z, beta, alpha, dt, ssm_a,
    conv_w, norm_w may be None."""
    _raise(lib().swq_gdn_step(_ptr(qkv), ld_qkv, _ptr(z), _ptr(beta), _ptr(alpha), _ptr(dt), _ptr(ssm_a),
                              _ptr(conv_w), _ptr(norm_w), _ptr(state), _ptr(conv_state), _ptr(y), rows, n_k_heads,
                              n_v_heads, key_head_dim, value_head_dim, conv_width, _stream(stream)))


def silu_mul(out, gate, up, n: int, rows: int = 1, ld: int | None = None, stream=None) -> None:
    _raise(lib().swq_silu_mul(_ptr(out), _ptr(gate), _ptr(up), n, rows, n if ld is None else ld, _stream(stream)))


def add(x, y, n: int, stream=None) -> None:
    _raise(lib().swq_add(_ptr(x), _ptr(y), n, _stream(stream)))


def embed(x, table, tokens, dim: int, vocab: int, rows: int = 1, stream=None) -> None:
    _raise(lib().swq_embed(_ptr(x), _ptr(table), _ptr(tokens), dim, vocab, rows, _stream(stream)))


def argmax(logits, n: int, rows: int, tokens, history=None, step=None, stream=None) -> None:
    _raise(lib().swq_argmax(_ptr(logits), n, rows, _ptr(tokens), _ptr(history), _ptr(step), _stream(stream)))


def decode_advance(pos, step=None, stream=None) -> None:
    _raise(lib().swq_decode_advance(_ptr(pos), _ptr(step), _stream(stream)))


def check(stream=None) -> None:
    """Synchronize and raise on a device-side wait timeout or CUDA error."""
    _raise(lib().swq_check(_stream(stream)))
