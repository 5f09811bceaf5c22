"""Generate the model-level golden vectors in this directory from the
reference itself.

Writes the tiny Llama GGUF files of tests/llama_gguf.py, loads each with
swllm.cpp's own Model (src/model.h compiled from source into
oracle/_ref/libswllm_model_ref.so, ``make -C oracle ref`` where the reference
tree is mounted), runs Model::forward teacher-forced over llama_gguf.TOKENS and
stores, per variant:

  golden_llama_<variant>.npz  sha256 -- of the GGUF file (the tests rebuild it
                                        and check it is the same file)
                              tokens [P] i32, logits [P, vocab] f32
                              config -- Model::load's hidden, ffn, layers,
                                        heads, kv_heads, head_dim, vocab,
                                        max_seq, rope_neox, rope_dim
                              config_f -- rms_norm_eps, rope_theta

usage: python tests/golden/make_golden_model.py [variant ...]   (default: all)
"""
from __future__ import annotations

import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path[:0] = [str(REPO), str(REPO / "swllm.cpp_b200"), str(REPO / "tests")]

import llama_gguf  # noqa: E402
from oracle.ref_model import RefModel  # noqa: E402


def main() -> None:
    with tempfile.TemporaryDirectory(dir=REPO / "tests" / "golden") as tmp:
        for variant in sys.argv[1:] or llama_gguf.VARIANTS:
            path = llama_gguf.write(Path(tmp) / f"{variant}.gguf", variant)
            m = RefModel(path)
            logits = np.stack([m.forward(tok, pos) for pos, tok in enumerate(llama_gguf.TOKENS)])
            c = m.config
            np.savez_compressed(
                HERE / f"golden_llama_{variant}.npz", sha256=np.array(llama_gguf.sha256(path)),
                tokens=np.array(llama_gguf.TOKENS, np.int32), logits=logits.astype(np.float32),
                config=np.array([c[k] for k in RefModel.CONFIG_I], np.int64),
                config_f=np.array([c["eps"], c["theta"]], np.float32))
            m.close()
            print(variant, logits.shape, llama_gguf.sha256(path)[:16])


if __name__ == "__main__":
    main()
