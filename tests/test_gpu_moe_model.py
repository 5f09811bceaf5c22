"""MoE decoder (swq.model.LlamaDecoder with a MoE config: attention as the
dense model, each FFN a swq.moe.MoEFFN of routed experts + a shared expert)
against the CPU model reference extended with the same MoE FFN
(oracle/model_ref.py, RefLlama._moe: the routing of oracle/moe_oracle.c and
the reference's quantized matmuls).

A 2-layer model: dim 256, 4 query / 2 kv heads of 64, 8 experts of 128 with
top-2 routing plus a shared expert of 128, vocab 300.  Decode logits must be
within MOE_LOGIT_TOL of the reference for the same tokens (the expert
products run through the grouped GEMV, whose activations are 16-bit fixed
point per 32 elements: a looser bound than the dense decode's 5e-4), and a
replayed CUDA graph must give the eager bits.
"""
import numpy as np
import pytest

from conftest import rel_l2
from swq import synth
from swq.model import LlamaConfig, LlamaDecoder, rope_freqs

pytestmark = pytest.mark.gpu

MOE_LOGIT_TOL = 2e-3


def _cfg(max_seq=32):
    t = synth
    types = {"wq": t.Q4_K, "wk": t.Q4_K, "wv": t.Q6_K, "wo": t.Q4_K, "output": t.Q6_K,
             "w_gate_exps": t.Q4_K, "w_up_exps": t.Q4_K, "w_down_exps": t.Q8_0,
             "w_gate_shexp": t.Q4_K, "w_up_shexp": t.Q4_K, "w_down_shexp": t.Q8_0}
    return LlamaConfig(n_layers=2, dim=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=128, vocab=300,
                       max_seq=max_seq, types=types, n_experts=8, top_k=2, expert_ffn=128, shared_ffn=128)


def _blocks(type_id, n, k, seed):
    if type_id in (synth.Q4_K, synth.Q5_K, synth.Q2_K, synth.Q3_K):
        return synth.centred_blocks(type_id, n, k, seed=seed)
    return synth.random_blocks(type_id, n, k, seed=seed)


def _weights(cfg, seed):
    rng = np.random.default_rng(seed)
    t = cfg.types
    layers = []
    for li in range(cfg.n_layers):
        L = {"attn_norm": (1 + 0.01 * rng.standard_normal(cfg.dim)).astype(np.float32),
             "ffn_norm": (1 + 0.01 * rng.standard_normal(cfg.dim)).astype(np.float32),
             "router": (0.02 * rng.standard_normal((cfg.n_experts, cfg.dim)) * 8).astype(np.float32)}
        for k, (n, kk) in cfg.shapes().items():
            L[k] = _blocks(t[k], n, kk, seed * 100 + li * 10 + len(L))
        for k, (n, kk) in cfg.moe_shapes().items():
            rows = n * cfg.n_experts if k.endswith("exps") else n
            L[k] = _blocks(t[k], rows, kk, seed * 100 + li * 10 + len(L))
        layers.append(L)
    return {"token_embd": rng.standard_normal((cfg.vocab, cfg.dim)).astype(np.float32),
            "output_norm": (1 + 0.01 * rng.standard_normal(cfg.dim)).astype(np.float32),
            "output": _blocks(t["output"], cfg.vocab, cfg.dim, seed * 100 + 99),
            "layers": layers}


def test_moe_decode_matches_reference(cuda):
    from oracle.model_ref import RefLlama
    cfg = _cfg()
    W = _weights(cfg, seed=3)
    rows = 2
    dec = LlamaDecoder(cfg, rows=rows, weights=W, moe_max_tokens=16)
    refs = [RefLlama(cfg, W, rope_freqs(cfg), cfg.max_seq) for _ in range(rows)]
    toks = [[5, 77, 123, 9, 200], [250, 1, 42, 42, 17]]
    for pos in range(len(toks[0])):
        dec.reset([toks[r][pos] for r in range(rows)], pos)
        dec.generate(1)
        dec.stream.synchronize()
        got = dec.logits.cpu().numpy()
        for r in range(rows):
            want = refs[r].forward(toks[r][pos], pos)
            assert rel_l2(got[r], want) <= MOE_LOGIT_TOL, (pos, r, rel_l2(got[r], want))
    import swq
    swq.check(dec.stream)


def test_moe_decode_graph_and_prefill(cuda):
    """A captured step replays the eager bits; a prefill of the same tokens
    ends at the decode's logits (tensor-core tolerance for the attention
    GEMMs of the prefill)."""
    torch = cuda
    cfg = _cfg()
    W = _weights(cfg, seed=4)
    a = LlamaDecoder(cfg, rows=2, weights=W, moe_max_tokens=8)
    b = LlamaDecoder(cfg, rows=2, weights_from=a)
    b.reset([3, 4], 0)
    b.capture()
    prompt = [[3, 10, 20, 30], [4, 11, 21, 31]]
    for pos in range(4):
        tok = [prompt[0][pos], prompt[1][pos]]
        a.reset(tok, pos)
        a.generate(1)
        b.reset(tok, pos)
        b.generate(1)
        a.stream.synchronize()
        b.stream.synchronize()
        assert torch.equal(a.logits, b.logits), pos
    last = a.logits.cpu().numpy().copy()
    c = LlamaDecoder(cfg, rows=2, weights_from=a)
    c.prefill(prompt)  # 8 rows: one MoE call of moe_max_tokens = 8
    c.stream.synchronize()
    assert rel_l2(c.logits.cpu().numpy(), last) <= 5e-2
    import swq
    swq.check(c.stream)
