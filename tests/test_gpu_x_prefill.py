"""Batched prefill on the GPU (swq_rope_kv_prefill, swq_attention_prefill,
LlamaDecoder.prefill).

* RoPE + KV append of M prompt rows against the decode step's swq_rope_kv
  run position by position (the same rotation, so within fp32 rounding).
* Causal attention against a float64 numpy restatement of the reference's
  per-token attention (src/model.h:329-361): 1e-5 relative L2.
* A whole prefill -- every projection one M-row tensor-core GEMM -- against
  the CPU restatement of Model::forward run token by token (the reference's
  prompt loop, src/main.cpp:284-287), at every prompt position: the
  tensor-core bound of the decode tests (TC_LOGIT_TOL), and the decode that
  follows the prefill against the same restatement.
"""
import numpy as np
import pytest

from conftest import rel_l2
from swq.model import LlamaDecoder, rope_freqs
from test_gpu_model import TC_LOGIT_TOL, _small, _weights

pytestmark = pytest.mark.gpu

ATT_TOL = 1e-5


def _attention_ref(q, kc, vc, pos0, P, S, H, Hkv, hd):
    """float64 causal attention: row m = s*P + p over positions 0..pos0+p."""
    q = q.astype(np.float64).reshape(S * P, H, hd)
    out = np.zeros((S * P, H, hd))
    for m in range(S * P):
        s, p = divmod(m, P)
        n = pos0 + p + 1
        for h in range(H):
            kvh = h // (H // Hkv)
            K = kc[s, :n, kvh * hd:(kvh + 1) * hd].astype(np.float64)
            V = vc[s, :n, kvh * hd:(kvh + 1) * hd].astype(np.float64)
            sc = K @ q[m, h] / np.sqrt(hd)
            w = np.exp(sc - sc.max())
            out[m, h] = (w / w.sum()) @ V
    return out.reshape(S * P, H * hd)


@pytest.mark.parametrize("S,P,pos0,H,Hkv,hd", [(1, 9, 0, 8, 2, 64), (3, 5, 4, 8, 8, 128), (2, 17, 11, 4, 1, 128),
                                                (1, 40, 0, 2, 2, 256), (2, 3, 0, 4, 2, 32),
                                                # tiled kernel: several query and key tiles, a
                                                # tile boundary, a context before the prompt
                                                (1, 200, 70, 8, 2, 128), (2, 130, 0, 4, 4, 64),
                                                (1, 64, 0, 2, 1, 128), (1, 65, 63, 4, 2, 64)])
@pytest.mark.parametrize("form", [3, 2, 1, 0], ids=["tensor-core-pairs", "tensor-core", "tiled-fp32", "warp-per-row"])
def test_attention_prefill_matches_numpy(cuda, S, P, pos0, H, Hkv, hd, form):
    """Every form of the causal attention (SWQ_OPT_PREFILL_ATTENTION) against
    float64; the tensor-core forms keep 22-bit operand pairs, within 1e-5."""
    torch = cuda
    import swq
    max_seq = pos0 + P + 3
    rng = np.random.default_rng(S * 100 + P)
    q = rng.standard_normal((S * P, H * hd), dtype=np.float32)
    kc = rng.standard_normal((S, max_seq, Hkv * hd), dtype=np.float32)
    vc = rng.standard_normal((S, max_seq, Hkv * hd), dtype=np.float32)
    d_out = torch.full((S * P, H * hd), float("nan"), device="cuda")
    old = swq.get_option(swq.OPT_PREFILL_ATTENTION)
    swq.set_option(swq.OPT_PREFILL_ATTENTION, form)
    try:
        swq.attention_prefill(d_out, torch.from_numpy(q).cuda(), torch.from_numpy(kc).cuda(),
                              torch.from_numpy(vc).cuda(), pos0, P, H, Hkv, hd, S, max_seq)
        swq.check()
    finally:
        swq.set_option(swq.OPT_PREFILL_ATTENTION, old)
    want = _attention_ref(q, kc, vc, pos0, P, S, H, Hkv, hd)
    assert rel_l2(d_out.cpu().numpy(), want) <= ATT_TOL


@pytest.mark.parametrize("form", [3, 2])
@pytest.mark.parametrize("hd", [64, 128])
def test_attention_prefill_tensor_core_dynamic_range(cuda, hd, form):
    """Tensor-core form: rows of q and k over many decades (each row its own
    scale), tiny and large values (v up to 1e6: scaled down below fp16's
    range, the softmax weights take the factor back), a non-finite q row
    (only its own outputs turn non-finite)."""
    torch = cuda
    import swq
    S, P, pos0, H, Hkv = 1, 150, 20, 4, 2
    max_seq = pos0 + P
    rng = np.random.default_rng(hd)
    q = (rng.standard_normal((S * P, H * hd)) * 10.0 ** rng.uniform(-4, 1, (S * P, 1))).astype(np.float32)
    kc = (rng.standard_normal((S, max_seq, Hkv * hd)) * 10.0 ** rng.uniform(-4, 1, (S, max_seq, 1))).astype(
        np.float32)
    vc = (rng.standard_normal((S, max_seq, Hkv * hd)) * 10.0 ** rng.uniform(-2, 6, (S, max_seq, 1))).astype(
        np.float32)
    q[7, :hd] = np.inf
    d_out = torch.full((S * P, H * hd), float("nan"), device="cuda")
    old = swq.get_option(swq.OPT_PREFILL_ATTENTION)
    swq.set_option(swq.OPT_PREFILL_ATTENTION, form)
    try:
        swq.attention_prefill(d_out, torch.from_numpy(q).cuda(), torch.from_numpy(kc).cuda(),
                              torch.from_numpy(vc).cuda(), pos0, P, H, Hkv, hd, S, max_seq)
        swq.check()
    finally:
        swq.set_option(swq.OPT_PREFILL_ATTENTION, old)
    got = d_out.cpu().numpy()
    assert not np.isfinite(got[7, :hd]).any()
    q[7, :hd] = 0.0
    want = _attention_ref(q, kc, vc, pos0, P, S, H, Hkv, hd)
    mask = np.ones_like(want, dtype=bool)
    mask[7, :hd] = False
    assert rel_l2(got[mask], want[mask]) <= ATT_TOL


@pytest.mark.parametrize("neox", [False, True])
def test_rope_kv_prefill_matches_decode_rope(cuda, neox):
    torch = cuda
    import swq
    S, P, pos0, qd, kvd, hd, max_seq = 2, 6, 3, 512, 128, 64, 16
    rng = np.random.default_rng(7)
    qk = torch.from_numpy(rng.standard_normal((S * P, qd + kvd), dtype=np.float32)).cuda()
    v = torch.from_numpy(rng.standard_normal((S * P, kvd), dtype=np.float32)).cuda()
    freqs = torch.from_numpy((1.0 / 10000.0 ** (np.arange(hd // 2) * 2.0 / hd)).astype(np.float32)).cuda()
    kc, vc = torch.zeros((S, max_seq, kvd), device="cuda"), torch.zeros((S, max_seq, kvd), device="cuda")
    q1 = qk.clone()
    swq.rope_kv_prefill(q1, q1[:, qd:], v, kc, vc, pos0, P, freqs, qd, kvd, hd, hd, neox, S, max_seq,
                        ldq=qd + kvd, ldk=qd + kvd, ldv=kvd)
    # the decode step's kernel, one position at a time for the S sequences
    kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
    q2 = qk.clone().view(S, P, qd + kvd)
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    for p in range(P):
        rows_q = q2[:, p].contiguous()
        rows_v = v.view(S, P, kvd)[:, p].contiguous()
        pos.fill_(pos0 + p)
        swq.rope_kv(rows_q, rows_q[:, qd:], rows_v, kc2, vc2, pos, freqs, qd, kvd, hd, hd, neox, S, max_seq,
                    ldq=qd + kvd, ldk=qd + kvd, ldv=kvd)
        q2[:, p] = rows_q
    swq.check()
    assert rel_l2(q1[:, :qd].cpu().numpy(), q2.view(S * P, -1)[:, :qd].cpu().numpy()) <= 1e-6
    assert rel_l2(kc.cpu().numpy(), kc2.cpu().numpy()) <= 1e-6
    assert torch.equal(vc, vc2)
    assert float(kc[:, :pos0].abs().sum()) == 0.0 and float(kc[:, pos0 + P:].abs().sum()) == 0.0


@pytest.mark.parametrize("rows,P", [(1, 6), (2, 5)])
def test_prefill_logits_match_reference(cuda, rows, P):
    """Every prompt position's logits against the restated forward run token by
    token; then the first decode step, which reads the prefilled cache."""
    from oracle.model_ref import RefLlama
    cfg = _small()
    W = _weights(cfg, seed=21)
    prompts = [[(37 * r + 11 * p + 3) % cfg.vocab for p in range(P)] for r in range(rows)]
    dec = LlamaDecoder(cfg, rows=rows, weights=W)
    every = dec.prefill(prompts, all_logits=True)
    dec.stream.synchronize()
    got = every.cpu().numpy()
    first = dec.tokens.cpu().numpy().copy()
    assert int(dec.pos.item()) == P and int(dec.step_no.item()) == 1
    dec.generate(1)
    dec.stream.synchronize()
    after = dec.logits.cpu().numpy()
    hist = dec.history[:2].cpu().numpy()
    assert int(dec.pos.item()) == P + 1
    for r in range(rows):
        ref = RefLlama(cfg, W, rope_freqs(cfg), cfg.max_seq)
        for p, tok in enumerate(prompts[r]):
            want = ref.forward(tok, p)
            assert rel_l2(got[r, p], want) <= TC_LOGIT_TOL, (r, p, rel_l2(got[r, p], want))
        assert first[r] == hist[0, r] == int(np.argmax(got[r, P - 1]))
        # K/V of the prompt come from the tensor-core projections: the same bound
        want = ref.forward(int(first[r]), P)
        assert rel_l2(after[r], want) <= TC_LOGIT_TOL, (r, rel_l2(after[r], want))
        assert hist[1, r] == int(np.argmax(after[r]))


@pytest.mark.parametrize("variant", ["mix", "tied", "neox", "bias", "qknorm", "hybrid"])
def test_gguf_prefill_matches_reference_logits(cuda, tmp_path, variant):
    """A GGUF file's prompt in one prefill against the logits of the
    reference's own Model::forward run token by token on the same file
    (tests/golden/golden_llama_<variant>.npz); "hybrid": a GatedDeltaNet
    layer, its recurrence one prompt position at a time."""
    import llama_gguf as LG
    from conftest import GOLDEN
    gold = np.load(GOLDEN / f"golden_llama_{variant}.npz")
    path = LG.write(tmp_path / "m.gguf", variant)
    assert LG.sha256(path) == str(gold["sha256"])
    dec = LlamaDecoder.from_gguf(path, rows=1)
    every = dec.prefill([gold["tokens"].tolist()], all_logits=True)
    dec.stream.synchronize()
    got = every[0].cpu().numpy()
    for p in range(got.shape[0]):
        assert rel_l2(got[p], gold["logits"][p]) <= TC_LOGIT_TOL, (p, rel_l2(got[p], gold["logits"][p]))
