"""Generate the golden vectors in this directory from the reference itself.

Runs swllm.cpp's own src/tensor.h, compiled from source into
oracle/_ref/libswllm_ref.so (``make -C oracle ref`` where the reference tree
is mounted), on seeded synthetic blocks and activations, and stores inputs and
outputs as small .npz files:

  golden_<FMT>.npz  blocks [N, row_bytes] u8, x [M, K] f32,
                    dequant [N*K] f32    -- reference dequantize()
                    gemv_ref [M, N] f32  -- Compute(Backend::CPU).matmul_transposed_q
                    gemv_dq [M, N] f32   -- reference dequantize() then the
                                            reference fp32 cpu_matmul_transposed
  golden_special_scales.npz
                    Q4_K/Q6_K/Q8_0 blocks whose fp16 d/dmin are zero, signed
                    zero, subnormal, max-normal, Inf and NaN-with-payload, with
                    the reference dequantize() output.

usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path[:0] = [str(REPO), str(REPO / "swllm.cpp_b200")]

import oracle  # noqa: E402
from swq import synth  # noqa: E402

SHAPES = {  # (N, K, M)
    "Q4_0": (16, 512, 2), "Q8_0": (16, 512, 2), "Q2_K": (16, 1024, 2), "Q3_K": (16, 1024, 2),
    "Q4_K": (16, 1024, 2), "Q5_K": (16, 1024, 2), "Q6_K": (16, 1024, 2),
}

SPECIAL_HALVES = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0xFBFF,
                  0x7C00, 0xFC00, 0x7E01, 0xFE3F, 0x3C00, 0x1234, 0x8001]


def main() -> None:
    if not oracle.ref_available():
        oracle.build(ref=True)
    for name, (N, K, M) in SHAPES.items():
        t = synth.IDS[name]
        blocks = synth.random_blocks(t, N, K, seed=1000 + t)
        x = synth.random_activations(M, K, seed=2000 + t)
        dq = oracle.ref_dequantize(t, blocks, N * K)
        gemv_ref = np.stack([oracle.ref_gemv(t, blocks, x[m], N, K) for m in range(M)])
        gemv_dq = np.stack([oracle.ref_gemv_f32(dq, x[m], N, K) for m in range(M)])
        np.savez_compressed(HERE / f"golden_{name}.npz", type=np.int32(t), N=np.int32(N), K=np.int32(K),
                            blocks=blocks, x=x, dequant=dq, gemv_ref=gemv_ref, gemv_dq=gemv_dq)
        print(f"golden_{name}.npz  N={N} K={K} M={M}")

    special = {}
    for name, fields in (("Q4_K", ("d", "dmin")), ("Q6_K", ("d",)), ("Q8_0", ("d",))):
        t = synth.IDS[name]
        qk, _ = synth.block_geometry(t)
        nblk = len(SPECIAL_HALVES)
        blocks = synth.random_blocks(t, 1, qk * nblk, seed=3000 + t)
        for i, h in enumerate(SPECIAL_HALVES):
            for f in fields:
                synth.set_block_scale(blocks, t, h if f == "d" else SPECIAL_HALVES[-1 - i], which=f, block=i)
        special[f"{name}_blocks"] = blocks
        special[f"{name}_dequant"] = oracle.ref_dequantize(t, blocks, qk * nblk)
    np.savez_compressed(HERE / "golden_special_scales.npz", **special)
    print("golden_special_scales.npz")


if __name__ == "__main__":
    main()
