"""The drop-in build on the CPU: the reference's own model code compiled in
its CUDA configuration with the one branch of Compute::matmul_transposed_q
(src/tensor.h:1214-1226) routed to libswq (oracle/make_dropin.py), linked to
libswq.so.  The GPU run of it is test_gpu_model.py's
test_reference_model_runs_on_libswq."""
import ctypes
from pathlib import Path

import pytest

from conftest import REPO

import oracle

REF_TENSOR_H = oracle.ref_src() / "tensor.h"


def test_derived_header_changes_only_the_matmul_branch():
    if not REF_TENSOR_H.exists():
        pytest.skip("reference sources not mounted")
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_dropin", REPO / "oracle" / "make_dropin.py")
    md = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(md)
    src = REF_TENSOR_H.read_text()
    out = md.derive(src)
    assert out.count(md.INCLUDE) == 1 and out.count(md.SWQ_BRANCH) == 1
    out = out.replace(md.INCLUDE, "", 1)
    i = out.index(md.SWQ_BRANCH)
    prefix, suffix = out[:i], out[i + len(md.SWQ_BRANCH):]
    # the derived file is the reference with exactly one span replaced ...
    assert src.startswith(prefix) and src.endswith(suffix)
    removed = src[len(prefix):len(src) - len(suffix)]
    # ... the CUDA branch (host dequantize + SGEMM) of Compute::matmul_transposed_q
    assert removed.startswith("#ifdef LLM_USE_CUDA") and removed.rstrip().endswith("#endif")
    assert removed.count("#if") == 1
    assert "dequantize(w.data, tmp.data()" in removed and "cuda_matmul_transposed_weight" in removed
    assert prefix.rstrip().splitlines()[-1].strip() == "const QuantWeight& w, int N, int K) {"


def test_dropin_library_calls_libswq():
    from oracle.ref_model import DROPIN_SO, dropin_available
    if not dropin_available():
        pytest.skip("drop-in build not made (needs the reference sources)")
    import swq
    d = ctypes.CDLL(str(DROPIN_SO))
    assert d.refm_load and d.refm_forward and d.dropin_errors() == 0
    # the drop-in's libswq is the very library the package loads
    assert ctypes.cast(d.swq_ctx_matmul_transposed_q, ctypes.c_void_p).value == \
        ctypes.cast(swq.lib().swq_ctx_matmul_transposed_q, ctypes.c_void_p).value


def test_dropin_fails_loudly_without_a_gpu(tmp_path, capfd):
    """No GPU: the reference's model loads, but every quantized matmul of its
    forward goes to libswq, which reports an error (printed and counted) --
    the drop-in has no silent CPU fallback for the seven formats."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present (the GPU test runs the drop-in)")
    from oracle.ref_model import RefModel, dropin_available
    if not dropin_available():
        pytest.skip("drop-in build not made (needs the reference sources)")
    import llama_gguf as LG
    m = RefModel(LG.write(tmp_path / "m.gguf", "mix"), dropin=True)
    before = m.dropin_errors()  # the count is per process
    m.forward(7, 0)
    # 2 layers x 7 projections + the LM head, every one refused
    assert m.dropin_errors() - before == 15
    assert "swq:" in capfd.readouterr().err
    m.close()
