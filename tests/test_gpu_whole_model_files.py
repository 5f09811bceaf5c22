"""Whole models from GGUF files on the GPU, against the reference's own logits.

The tiny Llama GGUF files of tests/llama_gguf.py ("mix": all seven formats,
a different type mix per layer, F32 embedding table; "tied": a Q8_0 embedding
table that is also the LM head; "neox": an architecture the reference runs
with neox RoPE), teacher-forced over the golden tokens, against
the logits the reference's CPU build produced (tests/golden/golden_llama_*.npz):

* LlamaDecoder.from_gguf -- libswq's device decode step;
* the drop-in -- the reference's own Model::forward built with its CUDA
  backend and the one matmul branch of tensor.h calling libswq.

Bound: LOGIT_TOL of the decode tests (5e-4 relative L2, the GEMV path's
per-projection errors compounding over the layers).  Q2_K matmuls follow the
reference's fused CPU routine, libswq's default order.  "bias" and "qknorm" carry the
optional q/k/v biases and q/k head norms; swq_qkv_bias_norm, which applies
them, is also checked alone against numpy (1e-6).
"""
import numpy as np
import pytest

from conftest import rel_l2
from swq.model import LlamaDecoder
from test_gpu_model import LOGIT_TOL, _teacher_forced

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("variant", ["mix", "tied", "neox", "bias", "qknorm", "hybrid"])
def test_gguf_model_matches_reference_logits(cuda, tmp_path, variant):
    """LlamaDecoder.from_gguf on a tiny GGUF file -- "mix": all seven formats,
    a different type mix per layer, F32 embedding table; "tied": a Q8_0
    embedding table that is also the LM head; "hybrid": a GatedDeltaNet layer
    then a full-attention layer -- teacher-forced, against the logits the
    reference's own Model::forward gave for the same file
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


# The reference's CUDA backend interface rotates with cuda_rope(q, k, q_dim,
# k_dim, head_dim, pos, theta) (src/tensor.h:27, Compute::rope), which has no
# neox argument: a CUDA build of the reference rotates interleaved pairs for
# every architecture.  The drop-in keeps that interface, so it is checked on
# the interleaved-RoPE files; the neox ones run through LlamaDecoder above.
@pytest.mark.parametrize("variant", ["mix", "tied"])
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


@pytest.mark.parametrize("which", ["bias", "norm", "both", "v_only"])
def test_qkv_bias_norm_matches_numpy(cuda, which):
    """swq_qkv_bias_norm on strided rows (q and k in one buffer) against the
    reference's order in numpy: q/k/v bias adds, then the RMSNorm of every q
    and k head with the shared [head_dim] weights (src/model.h:291-318)."""
    torch = cuda
    import swq
    rows, nh, nkv, hd, eps = 3, 8, 2, 64, 1e-5
    qd, kvd = nh * hd, nkv * hd
    rng = np.random.default_rng({"bias": 1, "norm": 2, "both": 3, "v_only": 4}[which])
    qk = rng.standard_normal((rows, qd + kvd), dtype=np.float32)
    v = rng.standard_normal((rows, kvd), dtype=np.float32)
    bq, bk, bv = (rng.standard_normal(n, dtype=np.float32) for n in (qd, kvd, kvd))
    qn, kn = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32), (1 + 0.1 * rng.standard_normal(hd)).astype(
        np.float32)
    use_b, use_n = which in ("bias", "both"), which in ("norm", "both")
    if which == "v_only":
        bq = bk = None
        use_b = False
    q_ref, k_ref, v_ref = qk[:, :qd].astype(np.float64), qk[:, qd:].astype(np.float64), v.astype(np.float64)
    if use_b:
        q_ref, k_ref = q_ref + bq, k_ref + bk
    if use_b or which == "v_only":
        v_ref = v_ref + bv
    if use_n:
        def hn(x, n, w):
            x = x.reshape(rows, n, hd)
            return (x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w).reshape(rows, n * hd)
        q_ref, k_ref = hn(q_ref, nh, qn), hn(k_ref, nkv, kn)
    d_qk, d_v = torch.from_numpy(qk).cuda(), torch.from_numpy(v).cuda()
    dev = lambda a, on: torch.from_numpy(a).cuda() if (on and a is not None) else None  # noqa: E731
    swq.qkv_bias_norm(d_qk, d_qk[:, qd:], d_v, dev(bq, use_b), dev(bk, use_b), dev(bv, use_b or which == "v_only"),
                      dev(qn, use_n), dev(kn, use_n), qd, kvd, hd, eps, rows, ldq=qd + kvd, ldk=qd + kvd, ldv=kvd)
    swq.check()
    got = d_qk.cpu().numpy()
    assert rel_l2(got[:, :qd], q_ref) <= 1e-6 and rel_l2(got[:, qd:], k_ref) <= 1e-6
    assert rel_l2(d_v.cpu().numpy(), v_ref) <= 1e-6
