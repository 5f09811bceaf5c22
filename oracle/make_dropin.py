"""Derive the drop-in build's tensor.h from the reference tree (TEST
INFRASTRUCTURE ONLY; the derived file goes to oracle/_ref/dropin/, which is
git-ignored, and is never committed).

The drop-in integration changes one branch of the reference: the
`#ifdef LLM_USE_CUDA` block of Compute::matmul_transposed_q
(src/tensor.h:1214-1226), which dequantizes on the host and multiplies with
cuBLAS, becomes a call into libswq on the GGUF blocks themselves
(swq_ctx_matmul_transposed_q).  Everything else in the reference -- GGUF
reader, Model::load, Model::forward, tokenizer -- is compiled unchanged from
the reference's own sources.  The build fails loudly if the branch is not
found exactly once.

usage: python oracle/make_dropin.py REF_SRC OUT_DIR
"""
from __future__ import annotations

import sys
from pathlib import Path

# The libswq context (created on first use; its weight cache is keyed by the
# host address of the GGUF blocks, so dropin_reset() destroys it when a model
# and its file buffer are freed) and the count of failed libswq calls (printed,
# counted, the process goes on).
INCLUDE = ('#include "swq.h"\ninline swq_ctx_t g_swq_dropin_ctx = nullptr;\n'
           'inline int g_swq_dropin_errors = 0;\n')

SWQ_BRANCH = r"""#ifdef LLM_USE_CUDA
        // libswq: the GGUF blocks go to the GPU as they are (uploaded once per
        // (pointer, type, N, K), then resident); out and x stay host fp32.
        if (backend == Backend::CUDA && swq_type_size(static_cast<int>(w.type)) > 0) {
            if (!g_swq_dropin_ctx && swq_ctx_create(0, &g_swq_dropin_ctx) != SWQ_OK)
                fprintf(stderr, "swq: %s\n", swq_last_error());
            const swq_status st = swq_ctx_matmul_transposed_q(g_swq_dropin_ctx, out, x, w.data,
                                                              static_cast<int>(w.type), N, K);
            if (st != SWQ_OK) {
                fprintf(stderr, "swq: %s (%s)\n", swq_status_string(st), swq_last_error());
                ++g_swq_dropin_errors;
            }
            return;
        }
#endif
"""


def derive(src: str) -> str:
    lines = src.splitlines(keepends=True)
    heads = [i for i, ln in enumerate(lines) if "void matmul_transposed_q(float* out" in ln]
    if len(heads) != 1:
        raise SystemExit(f"make_dropin: {len(heads)} definitions of matmul_transposed_q found, expected 1")
    i = heads[0]
    start = next(j for j in range(i, min(i + 6, len(lines))) if lines[j].strip() == "#ifdef LLM_USE_CUDA")
    end = next(j for j in range(start + 1, len(lines)) if lines[j].strip().startswith("#"))
    if lines[end].strip() != "#endif":
        raise SystemExit(f"make_dropin: unexpected directive in the CUDA branch: {lines[end].strip()}")
    if "cuda_matmul_transposed_weight" not in "".join(lines[start:end]):
        raise SystemExit("make_dropin: the CUDA branch does not look like the host-dequant + SGEMM path")
    guard = next(j for j, ln in enumerate(lines) if ln.startswith("#define LLM_TENSOR_H"))
    out = lines[:guard + 1] + [INCLUDE] + lines[guard + 1:start] + [SWQ_BRANCH] + lines[end + 1:]
    return "".join(out)


def main() -> None:
    ref_src, out_dir = Path(sys.argv[1]), Path(sys.argv[2])
    out_dir.mkdir(parents=True, exist_ok=True)
    (out_dir / "tensor.h").write_text(derive((ref_src / "tensor.h").read_text()))


if __name__ == "__main__":
    main()
