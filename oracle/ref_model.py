"""ctypes wrapper of the reference's GGUF reader and Model, compiled from
source by ``make -C oracle ref`` (_ref/libswllm_model_ref.so, model_shim.cpp).
TEST INFRASTRUCTURE ONLY.

``RefGGUF(path)``  -- GGUFFile::load (src/gguf.h:238-257) and its lookups.
``RefModel(path)`` -- Model::load (src/model.h:220-255) on the CPU backend;
                      ``forward(token, pos)`` is Model::forward (:257-543).
``RefModel(path, dropin=True)`` -- the same reference code in its CUDA build
                      with Compute::matmul_transposed_q routed to libswq
                      (_ref/libswllm_dropin.so, make_dropin.py): the drop-in.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import HERE

MODEL_REF_SO = HERE / "_ref" / "libswllm_model_ref.so"
DROPIN_SO = HERE / "_ref" / "libswllm_dropin.so"
_libs: dict = {}


def model_ref_available() -> bool:
    return MODEL_REF_SO.exists()


def dropin_available() -> bool:
    return DROPIN_SO.exists()


def _l(dropin: bool = False) -> ctypes.CDLL:
    path = DROPIN_SO if dropin else MODEL_REF_SO
    if path not in _libs:
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (needs the reference sources)")
        lib = ctypes.CDLL(str(path))
        vp, cp, ull = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_ulonglong
        lib.refg_open.restype = vp
        lib.refg_open.argtypes = [cp]
        lib.refg_close.argtypes = [vp]
        lib.refg_header.argtypes = [vp, ctypes.POINTER(ull)]
        lib.refg_tensor.restype = ctypes.c_int
        lib.refg_tensor.argtypes = [vp, cp, ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_uint),
                                    ctypes.POINTER(ull), ctypes.POINTER(ull), ctypes.POINTER(ull)]
        lib.refg_tensor_file_offset.restype = ctypes.c_longlong
        lib.refg_tensor_file_offset.argtypes = [vp, cp]
        lib.refg_get_i64.restype = ctypes.c_longlong
        lib.refg_get_i64.argtypes = [vp, cp, ctypes.c_longlong]
        lib.refg_get_f64.restype = ctypes.c_double
        lib.refg_get_f64.argtypes = [vp, cp, ctypes.c_double]
        lib.refg_get_str.restype = ctypes.c_longlong
        lib.refg_get_str.argtypes = [vp, cp, ctypes.c_char_p, ctypes.c_longlong]
        lib.refg_array_len.restype = ctypes.c_longlong
        lib.refg_array_len.argtypes = [vp, cp]
        lib.refm_load.restype = vp
        lib.refm_load.argtypes = [cp, ctypes.c_int]
        lib.refm_free.argtypes = [vp]
        lib.refm_config_i.argtypes = [vp, ctypes.POINTER(ctypes.c_int)]
        lib.refm_config_f.argtypes = [vp, ctypes.POINTER(ctypes.c_float)]
        lib.refm_forward.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]
        lib.refm_clear.argtypes = [vp]
        _libs[path] = lib
    return _libs[path]


class RefGGUF:
    def __init__(self, path):
        self.h = _l().refg_open(str(path).encode())
        if not self.h:
            raise ValueError(f"reference GGUFFile::load failed on {path}")
        hdr = (ctypes.c_ulonglong * 5)()
        _l().refg_header(self.h, hdr)
        self.version, self.tensor_count, self.metadata_kv_count, self.alignment, self.data_offset = list(hdr)

    def close(self):
        if self.h:
            _l().refg_close(self.h)
            self.h = None

    __del__ = close

    def tensor(self, name: str):
        """(type, n_dims, dims[4], offset, num_bytes, file offset) or None."""
        t, nd = ctypes.c_uint(), ctypes.c_uint()
        dims = (ctypes.c_ulonglong * 4)()
        off, nb = ctypes.c_ulonglong(), ctypes.c_ulonglong()
        if not _l().refg_tensor(self.h, name.encode(), ctypes.byref(t), ctypes.byref(nd), dims, ctypes.byref(off),
                                ctypes.byref(nb)):
            return None
        return (t.value, nd.value, tuple(dims), off.value, nb.value,
                _l().refg_tensor_file_offset(self.h, name.encode()))

    def get_i64(self, key: str, default: int = 0) -> int:
        return _l().refg_get_i64(self.h, key.encode(), default)

    def get_f64(self, key: str, default: float = 0.0) -> float:
        return _l().refg_get_f64(self.h, key.encode(), default)

    def get_str(self, key: str) -> str:
        n = _l().refg_get_str(self.h, key.encode(), None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        _l().refg_get_str(self.h, key.encode(), buf, n + 1)
        return buf.raw[:n].decode("utf-8", errors="surrogateescape")

    def array_len(self, key: str) -> int:
        return _l().refg_array_len(self.h, key.encode())


class RefModel:
    CONFIG_I = ("hidden", "ffn", "layers", "heads", "kv_heads", "head_dim", "vocab", "max_seq", "rope_neox",
                "rope_dim")

    def __init__(self, path, context_override: int = 0, dropin: bool = False):
        self.lib, self.dropin = _l(dropin), dropin
        self.h = self.lib.refm_load(str(path).encode(), context_override)
        if not self.h:
            raise ValueError(f"reference Model::load failed on {path}")
        ci = (ctypes.c_int * 10)()
        cf = (ctypes.c_float * 2)()
        self.lib.refm_config_i(self.h, ci)
        self.lib.refm_config_f(self.h, cf)
        self.config = dict(zip(self.CONFIG_I, list(ci)))
        self.config["eps"], self.config["theta"] = float(cf[0]), float(cf[1])

    def close(self):
        if self.h:
            self.lib.refm_free(self.h)
            self.h = None
            if self.dropin:  # libswq's weights were keyed by the freed file buffer
                self.lib.dropin_reset()

    __del__ = close

    def forward(self, token: int, pos: int) -> np.ndarray:
        out = np.zeros(self.config["vocab"], np.float32)
        self.lib.refm_forward(self.h, token, pos, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        return out

    def clear(self) -> None:
        self.lib.refm_clear(self.h)

    def dropin_errors(self) -> int:
        """libswq calls of the drop-in build that returned an error."""
        return self.lib.dropin_errors()
