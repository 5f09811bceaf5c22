"""Host-array mirror of the reference's compute interface for this path.

``QuantWeight`` / ``Compute.matmul_transposed_q`` / ``dequantize`` keep the
reference's names and argument meaning (src/tensor.h:451, 507-511, 1212):
``out`` and ``x`` are host fp32 arrays, the weight is a host buffer of GGUF
blocks plus its GGMLType.  The CUDA backend uploads each weight once and keeps
it resident (the reference's GPUWeightCache, src/cuda_kernels.cu:88-127, keyed
here by host address, type and shape), then runs the fused libswq kernel.
Errors raise ``SwqError`` (the reference prints to stderr instead).
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass

import numpy as np

from .lib import _raise, lib


class Backend(enum.Enum):
    CUDA = "CUDA"   # src/tensor.h:515-518; the CPU backend is not part of this library


@dataclass
class QuantWeight:
    """src/tensor.h:507-511: non-owning view of GGUF blocks and their type."""
    data: np.ndarray
    type: int

    def valid(self) -> bool:
        return self.data is not None


def _host_ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Compute:
    """Compute(Backend::CUDA) for the quantized matmul path on one GPU."""

    def __init__(self, backend: Backend = Backend.CUDA, device: int = 0):
        if backend is not Backend.CUDA:
            raise ValueError("only the CUDA backend exists in this library")
        self.backend = backend
        self._ctx = ctypes.c_void_p()
        _raise(lib().swq_ctx_create(device, ctypes.byref(self._ctx)))

    def close(self) -> None:
        if self._ctx:
            lib().swq_ctx_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter teardown order
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @staticmethod
    def _f32(a: np.ndarray, name: str) -> np.ndarray:
        if not (isinstance(a, np.ndarray) and a.dtype == np.float32 and a.flags.c_contiguous):
            raise TypeError(f"{name} must be a C-contiguous float32 numpy array")
        return a

    def matmul_transposed_q(self, out: np.ndarray, x: np.ndarray, w: QuantWeight, N: int, K: int) -> None:
        """out[N] = W[N x K] . x[K]  (src/tensor.h:1212)."""
        self._f32(out, "out")
        self._f32(x, "x")
        if out.size < N or x.size < K:
            raise ValueError("out/x smaller than N/K")
        blocks = np.ascontiguousarray(w.data, dtype=np.uint8)
        _raise(lib().swq_ctx_matmul_transposed_q(self._ctx, _host_ptr(out), _host_ptr(x),
                                                 _host_ptr(blocks), w.type, N, K))

    def matmul_q_batched(self, Y: np.ndarray, X: np.ndarray, w: QuantWeight, M: int, N: int, K: int) -> None:
        """Y[M x N] = X[M x K] . W^T: M calls of matmul_transposed_q in one launch."""
        self._f32(Y, "Y")
        self._f32(X, "X")
        if Y.size < M * N or X.size < M * K:
            raise ValueError("Y/X smaller than M*N/M*K")
        blocks = np.ascontiguousarray(w.data, dtype=np.uint8)
        _raise(lib().swq_ctx_matmul_q_batched(self._ctx, _host_ptr(Y), _host_ptr(X),
                                              _host_ptr(blocks), w.type, M, N, K))

    def dequantize(self, src: np.ndarray, dst: np.ndarray, n: int, type_id: int) -> None:
        self._f32(dst, "dst")
        blocks = np.ascontiguousarray(src, dtype=np.uint8)
        _raise(lib().swq_ctx_dequantize(self._ctx, _host_ptr(blocks), _host_ptr(dst), n, type_id))

    def evict(self, w: QuantWeight) -> None:
        _raise(lib().swq_ctx_evict(self._ctx, _host_ptr(w.data)))

    def resident_bytes(self) -> int:
        return int(lib().swq_ctx_resident_bytes(self._ctx))


_default: Compute | None = None


def dequantize(src: np.ndarray, dst: np.ndarray, n: int, type_id: int) -> None:
    """dequantize(src, dst, n, type) (src/tensor.h:451) on the GPU, host arrays."""
    global _default
    if _default is None:
        _default = Compute()
    _default.dequantize(src, dst, n, type_id)
