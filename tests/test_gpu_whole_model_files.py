"""Whole models from GGUF files on the GPU, against the reference's own logits.

The tiny Llama GGUF files of tests/llama_gguf.py ("mix": all seven formats,
a different type mix per layer, F32 embedding table; "tied": a Q8_0 embedding
table that is also the LM head; "neox": an architecture the reference runs
with neox RoPE), teacher-forced over the golden tokens, against
the logits the reference's CPU build produced (tests/golden/golden_llama_*.npz):

* LlamaDecoder.from_gguf -- libswq's device decode step;
* the drop-in -- the reference's own Model::forward built with its CUDA
  backend and the one matmul branch of tensor.h calling libswq.

Bound: LOGIT_TOL of the decode tests (2e-3 relative L2, the GEMV path's 16-bit
activations compounding over the layers).
"""
import numpy as np
import pytest

from conftest import rel_l2
from swq.model import LlamaDecoder
from test_gpu_model import LOGIT_TOL, _teacher_forced

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("variant", ["mix", "tied", "neox"])
def test_gguf_model_matches_reference_logits(cuda, tmp_path, variant):
    """LlamaDecoder.from_gguf on a tiny GGUF file -- "mix": all seven formats,
    a different type mix per layer, F32 embedding table; "tied": a Q8_0
    embedding table that is also the LM head -- teacher-forced, against the
    logits the reference's own Model::forward gave for the same file
    (tests/golden/golden_llama_<variant>.npz)."""
    import llama_gguf as LG
    from conftest import GOLDEN
    gold = np.load(GOLDEN / f"golden_llama_{variant}.npz")
    path = LG.write(tmp_path / "m.gguf", variant)
    assert LG.sha256(path) == str(gold["sha256"])
    dec = LlamaDecoder.from_gguf(path, rows=1)
    toks = gold["tokens"].tolist()
    got = _teacher_forced(dec, 1, toks)
    for pos in range(len(toks)):
        want = gold["logits"][pos]
        assert rel_l2(got[pos, 0], want) <= LOGIT_TOL, (pos, rel_l2(got[pos, 0], want))
        top2 = np.sort(want)[-2:]
        if top2[1] - top2[0] > 1e-2 * np.abs(want).max():
            assert int(np.argmax(got[pos, 0])) == int(np.argmax(want)), pos


@pytest.mark.parametrize("variant", ["mix", "tied", "neox"])
def test_reference_model_runs_on_libswq(cuda, tmp_path, variant):
    """The drop-in: the reference's own Model::load / Model::forward, built with
    its CUDA backend and the one matmul branch of tensor.h calling
    swq_ctx_matmul_transposed_q (oracle/_ref/libswllm_dropin.so), on the tiny
    GGUF files, against the logits of the reference's CPU build."""
    from oracle.ref_model import RefModel, dropin_available
    if not dropin_available():
        pytest.skip("drop-in build not made (needs the reference sources where it is built)")
    import llama_gguf as LG
    from conftest import GOLDEN
    gold = np.load(GOLDEN / f"golden_llama_{variant}.npz")
    path = LG.write(tmp_path / "m.gguf", variant)
    m = RefModel(path, dropin=True)
    for pos, tok in enumerate(gold["tokens"].tolist()):
        got = m.forward(tok, pos)
        assert m.dropin_errors() == 0, "a libswq call of the drop-in failed (printed on stderr)"
        want = gold["logits"][pos]
        assert rel_l2(got, want) <= LOGIT_TOL, (pos, rel_l2(got, want))
    m.close()
