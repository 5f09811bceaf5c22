"""Python loader for the test oracle (TEST INFRASTRUCTURE ONLY).

Two CPU implementations of swllm.cpp's quantized-weight path, both loaded with
ctypes:

* ``liboracle.so`` -- ``swq_oracle.c``, a plain-C restatement of the reference's
  dequantizers and fused GEMVs (src/tensor.h:136-1025) with the same fp32
  expression trees and accumulation order.
* ``_ref/libswllm_ref.so`` -- the reference's own src/tensor.h compiled from
  source (``make -C oracle ref``); present only where it was built.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline/reference
arm import this package; the product library never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libswllm_ref.so"

# GGMLType ids and block geometry, src/gguf.h:18-40, 60-118.
Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 2, 8, 10, 11, 12, 13, 14
FORMATS = {
    "Q4_0": (Q4_0, 32, 18),
    "Q8_0": (Q8_0, 32, 34),
    "Q2_K": (Q2_K, 256, 84),
    "Q3_K": (Q3_K, 256, 110),
    "Q4_K": (Q4_K, 256, 144),
    "Q5_K": (Q5_K, 256, 176),
    "Q6_K": (Q6_K, 256, 210),
}
TYPE_IDS = {name: t for name, (t, _, _) in FORMATS.items()}
BLOCK = {t: (qk, bb) for _, (t, qk, bb) in FORMATS.items()}

_f32p = ctypes.POINTER(ctypes.c_float)


def build(ref: bool = True) -> None:
    """Compile liboracle.so (and _ref when the reference tree is present)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "liboracle.so"], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref"], check=True)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


class _Lib:
    def __init__(self, path: Path):
        self.path = path
        self.lib = ctypes.CDLL(str(path))


_oracle = None
_ref = None


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not ORACLE_SO.exists():
            build(ref=False)
        lib = ctypes.CDLL(str(ORACLE_SO))
        lib.oracle_dequantize.restype = ctypes.c_int
        lib.oracle_dequantize.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        for fn in (lib.oracle_matmul_transposed_q, lib.oracle_matmul_transposed_q_format_order):
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                           ctypes.c_int, ctypes.c_int]
        lib.oracle_matmul_q_batched.restype = ctypes.c_int
        lib.oracle_matmul_q_batched.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_int]
        lib.oracle_fp16_to_fp32.restype = ctypes.c_float
        lib.oracle_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        lib.oracle_type_size.restype = ctypes.c_size_t
        lib.oracle_block_size.restype = ctypes.c_size_t
        lib.oracle_type_size.argtypes = [ctypes.c_int]
        lib.oracle_block_size.argtypes = [ctypes.c_int]
        lib.oracle_set_threads.restype = ctypes.c_int
        lib.oracle_set_threads.argtypes = [ctypes.c_int]
        lib.oracle_q3k_scales.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.oracle_get_scale_min_k4.argtypes = [ctypes.c_int, ctypes.c_void_p,
                                                ctypes.c_void_p, ctypes.c_void_p]
        vp, i32 = ctypes.c_void_p, ctypes.c_int
        lib.oracle_moe_router_logits.argtypes = [vp, vp, i32, i32, i32, vp]
        lib.oracle_moe_topk_softmax.argtypes = [vp, i32, i32, i32, vp, vp]
        lib.oracle_moe_sort.restype = ctypes.c_int
        lib.oracle_moe_sort.argtypes = [vp, i32, i32, vp, vp, vp]
        lib.oracle_moe_combine.argtypes = [vp, vp, vp, i32, i32, i32, vp, i32]
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return REF_SO.exists()


def ref_lib() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} not built (needs the reference sources)")
        lib = ctypes.CDLL(str(REF_SO))
        lib.ref_dequantize.restype = None
        lib.ref_dequantize.argtypes = [ctypes.c_uint, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong]
        lib.ref_matmul_transposed_q.restype = None
        lib.ref_matmul_transposed_q.argtypes = [ctypes.c_uint, ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        lib.ref_matmul_transposed.restype = None
        lib.ref_matmul_transposed.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_int, ctypes.c_int]
        lib.ref_fp16_to_fp32.restype = ctypes.c_float
        lib.ref_fp16_to_fp32.argtypes = [ctypes.c_ushort]
        lib.ref_type_size.restype = ctypes.c_size_t
        lib.ref_type_size.argtypes = [ctypes.c_uint]
        lib.ref_block_size.restype = ctypes.c_size_t
        lib.ref_block_size.argtypes = [ctypes.c_uint]
        lib.ref_max_threads.restype = ctypes.c_int
        lib.ref_set_threads.argtypes = [ctypes.c_int]
        _ref = lib
    return _ref


def _check_w(blocks: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    return b


# ---- oracle (C restatement) -------------------------------------------------

def dequantize(type_id: int, blocks: np.ndarray, n: int) -> np.ndarray:
    b = _check_w(blocks)
    out = np.zeros(n, dtype=np.float32)
    rc = oracle_lib().oracle_dequantize(type_id, _ptr(b), _ptr(out), n)
    if rc != 0:
        raise ValueError(f"oracle: unsupported type {type_id}")
    return out


def gemv(type_id: int, blocks: np.ndarray, x: np.ndarray, N: int, K: int,
         format_order: bool = False) -> np.ndarray:
    """out[N] = W . x, as Compute::matmul_transposed_q (src/tensor.h:1212) on
    the reference's CPU backend.  ``format_order`` selects, for Q2_K only, the
    element order of dequantize_q2_k (src/tensor.h:232-265) instead of the
    fused routine's (src/tensor.h:935-945); every other format has one order."""
    b = _check_w(blocks)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    assert xx.size == K
    out = np.zeros(N, dtype=np.float32)
    fn = (oracle_lib().oracle_matmul_transposed_q_format_order if format_order
          else oracle_lib().oracle_matmul_transposed_q)
    rc = fn(type_id, _ptr(out), _ptr(xx), _ptr(b), N, K)
    if rc != 0:
        raise ValueError(f"oracle: unsupported type {type_id}")
    return out


def gemm(type_id: int, blocks: np.ndarray, X: np.ndarray, M: int, N: int, K: int,
         format_order: bool = False) -> np.ndarray:
    """Y[M x N] = X . W^T: M calls of gemv (the reference has no batched
    quantized path), same ``format_order`` meaning."""
    b = _check_w(blocks)
    XX = np.ascontiguousarray(X, dtype=np.float32).reshape(M, K)
    Y = np.zeros((M, N), dtype=np.float32)
    rc = oracle_lib().oracle_matmul_q_batched(type_id, _ptr(Y), _ptr(XX), _ptr(b), M, N, K,
                                              1 if format_order else 0)
    if rc != 0:
        raise ValueError(f"oracle: unsupported type {type_id}")
    return Y


def fp16_to_fp32(h: int) -> float:
    return oracle_lib().oracle_fp16_to_fp32(h)


def set_threads(n: int) -> int:
    return oracle_lib().oracle_set_threads(n)


# ---- the reference itself, compiled from source ------------------------------

def ref_dequantize(type_id: int, blocks: np.ndarray, n: int) -> np.ndarray:
    b = _check_w(blocks)
    out = np.zeros(n, dtype=np.float32)
    ref_lib().ref_dequantize(type_id, _ptr(b), _ptr(out), n)
    return out


def ref_gemv(type_id: int, blocks: np.ndarray, x: np.ndarray, N: int, K: int) -> np.ndarray:
    """Compute(Backend::CPU).matmul_transposed_q, src/tensor.h:1212."""
    b = _check_w(blocks)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(N, dtype=np.float32)
    ref_lib().ref_matmul_transposed_q(type_id, _ptr(out), _ptr(xx), _ptr(b), N, K)
    return out


def ref_gemv_f32(w: np.ndarray, x: np.ndarray, N: int, K: int) -> np.ndarray:
    ww = np.ascontiguousarray(w, dtype=np.float32)
    xx = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(N, dtype=np.float32)
    ref_lib().ref_matmul_transposed(_ptr(out), _ptr(xx), _ptr(ww), N, K)
    return out


def ref_set_threads(n: int) -> None:
    ref_lib().ref_set_threads(n)


def ref_src() -> Path:
    """Directory of the reference's sources: $REF_SRC, else the default the
    oracle's Makefile builds _ref/ from."""
    env = os.environ.get("REF_SRC")
    if env:
        return Path(env)
    for ln in (Path(__file__).resolve().parent / "Makefile").read_text().splitlines():
        if ln.startswith("REF_SRC ?="):
            return Path(ln.split("?=", 1)[1].strip())
    return Path("reference-sources-not-configured")


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


# ---------------------------------------------------------------- MoE routing
# The reference has no MoE forward; moe_oracle.c states the routing as libswq
# defines it (parity for routing is unpinned by the reference).

def moe_router_logits(W: np.ndarray, X: np.ndarray) -> np.ndarray:
    """logits [T, E] in float64 of the fp32 router W [E, H] on X [T, H]."""
    W = np.ascontiguousarray(W, dtype=np.float32)
    X = np.ascontiguousarray(X, dtype=np.float32)
    T, H = X.shape
    E = W.shape[0]
    out = np.empty((T, E), dtype=np.float64)
    oracle_lib().oracle_moe_router_logits(_ptr(W), _ptr(X), T, E, H, _ptr(out))
    return out


def moe_topk_softmax(logits: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """(ids [T, k] int32, weights [T, k] float32) from fp32 logits [T, E]."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    ids = np.empty((T, k), dtype=np.int32)
    w = np.empty((T, k), dtype=np.float32)
    oracle_lib().oracle_moe_topk_softmax(_ptr(logits), T, E, k, _ptr(ids), _ptr(w))
    return ids, w


def moe_sort(ids: np.ndarray, n_experts: int) -> tuple[np.ndarray, np.ndarray, np.ndarray, int]:
    """(offsets [E+1], sorted [rows], prow [P], pairs left out) of the pairs ids (any shape)."""
    flat = np.ascontiguousarray(ids, dtype=np.int32).reshape(-1)
    P = flat.size
    offsets = np.empty(n_experts + 1, dtype=np.int32)
    sorted_ = np.full(max(P, 1), -1, dtype=np.int32)
    prow = np.empty(max(P, 1), dtype=np.int32)
    bad = oracle_lib().oracle_moe_sort(_ptr(flat), P, n_experts, _ptr(offsets), _ptr(sorted_), _ptr(prow))
    return offsets, sorted_[:offsets[-1]], prow[:P], int(bad)


def moe_combine(Ys: np.ndarray, prow: np.ndarray, w: np.ndarray, T: int, k: int, H: int,
                Y0: np.ndarray | None = None) -> np.ndarray:
    """Y [T, H] = (Y0 or 0) + sum_j w[t, j] * Ys[prow[t*k + j]] with one fmaf per slot."""
    Ys = np.ascontiguousarray(Ys, dtype=np.float32)
    prow = np.ascontiguousarray(prow, dtype=np.int32).reshape(-1)
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    Y = np.zeros((T, H), dtype=np.float32) if Y0 is None else np.array(Y0, dtype=np.float32, copy=True)
    oracle_lib().oracle_moe_combine(_ptr(Ys), _ptr(prow), _ptr(w), T, k, H, _ptr(Y), 0 if Y0 is None else 1)
    return Y


def ep_layout(ids_per_rank: list, n_experts: int, world: int) -> list[dict]:
    """Expert-parallel placement of every rank's pairs (ids_per_rank[s] is
    rank s's [T_s, k] global expert ids): for each rank d, its local expert
    offsets `loff` and the (source, slot) of each received row, where slot is
    the pair's position in its source's stable sort by expert.  Rows of a
    local expert come from source 0, 1, ... in turn, each source's pairs in
    pair order."""
    el = n_experts // world
    sorts = [moe_sort(ids, n_experts) for ids in ids_per_rank]
    out = []
    for d in range(world):
        loff = [0]
        tags = []
        for le in range(el):
            e = d * el + le
            for s, (offs, _, _, _) in enumerate(sorts):
                tags.extend((s, i) for i in range(offs[e], offs[e + 1]))
            loff.append(len(tags))
        out.append({"loff": np.array(loff, dtype=np.int32), "tags": tags})
    return out
