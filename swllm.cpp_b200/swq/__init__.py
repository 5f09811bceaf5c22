"""swq -- B200 (sm_100a) quantized-weight matmul for swllm.cpp models.

Python host side over the C ABI of ``libswq.so`` (declared in include/swq.h).
It mirrors the reference's interface for this path (src/tensor.h):

* ``QuantWeight`` (src/tensor.h:507-511), ``Compute.matmul_transposed_q``
  (src/tensor.h:1212) and ``dequantize`` (src/tensor.h:451) with host arrays;
* device-pointer entry points ``dequant``, ``gemv``, ``gemm`` for callers that
  keep weights and activations resident on the GPU (torch tensors or raw
  pointers).

Around them: ``swq.model.LlamaDecoder`` (device decode step and batched
prefill, CUDA graphs, tensor parallelism; ``from_gguf`` loads a model file),
``swq.gguf`` (GGUF reader and writer, read as the reference's GGUFFile,
src/gguf.h), ``swq.parallel`` / ``swq.comm`` (parallel layers, expert-parallel
MoE, peer all-reduce).

All arithmetic runs in the CUDA kernels of libswq.  There is no CPU fallback:
if the library is missing or the GPU is not an sm_100 part, calls raise.
"""
from __future__ import annotations

from .lib import (  # noqa: F401
    Q2_K, Q3_K, Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, TYPES, TYPE_NAMES,
    OPT_EARLY_WEIGHT_PREFETCH, OPT_GEMV_MAX_M, OPT_Q2K_REFERENCE_CPU_ORDER, OPT_TENSOR_CORE_GEMM,
    OPT_TENSOR_CORE_MIN_M, OPT_GEMV_SMEM_KB, OPT_GEMV_STAGE_KB, OPT_GEMV_CTAS_PER_SM, OPT_GEMV_FP32_ACT, OPT_GEMV_INT_MMA,
    OPT_GEMV_BATCH_MAX_M, OPT_GEMV_BATCH_TABLE_KB, OPT_GEMV_BATCH_GROUP, OPT_PREFILL_ATTENTION,
    ACT_NONE, ACT_RMSNORM, ACT_SWIGLU,
    add, add_rmsnorm, argmax, attention_decode, attention_prefill, attention_workspace_bytes, decode_advance, embed,
    gdn_step,
    qkv_bias_norm, rmsnorm, rope_kv, rope_kv_prefill, silu_mul,
    GEMM_NOALLOC_MAX_X_ELEMS, SwqError, Status, block_size, build, check, dequant, exported_symbols, gemm,
    gemm_act, gemm_act_ws, gemm_noalloc, gemm_workspace_bytes, gemv, grouped_gemm, grouped_gemv, grouped_matmul, grouped_matmul_stacked,
    moe_combine, moe_gather, moe_router, moe_sort,
    get_option, header_symbols, lib, lib_path, set_option, type_size,
)
from .compute import Backend, Compute, QuantWeight, dequantize  # noqa: F401
