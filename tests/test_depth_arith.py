"""Model-level accuracy of each projection form at depth, on the CPU: the
restated decode forward (oracle/model_ref.py, pinned to the reference's own
Model::forward, src/model.h:257-543) with its quantized matmuls replaced by
numpy emulations of the device kernels' arithmetic (test_gemv_arith.py,
test_gemm_tc_arith.py), against the same forward with the reference's matmul.

Llama-shaped Q4_K_M models (dim 512, 8 / 2 heads of 64, FFN 1024, vocab
1000, centred blocks as a quantizer makes them) of 2 to 80 layers,
teacher-forced over four positions; largest logit rel-L2:

  layers   single-row GEMV   batched GEMV   tensor-core GEMM (fp16 operands)
     2        2.4e-6            2.5e-6          2.9e-3
     8        5.9e-6            5.6e-6          1.2e-2
    32        9.9e-6            1.05e-5         1.25e-2
    80        3.0e-5            2.7e-5          2.4e-2

The K-quant GEMV forms (every decode of up to 16 rows) stay two orders of
magnitude inside the GPU tests' 5e-4 even at the 70B model's depth; the
tensor-core form (prefill, decode of 17 rows or more) grows to a few 1e-2.
The emulations sum in float64, so the kernels' fp32 sums come on top
(the GPU tests measure those at 4 layers)."""
import numpy as np
import pytest

from conftest import rel_l2

TOKS = [11, 500, 7, 42]


def _forms():
    import test_gemm_tc_arith as TA
    import test_gemv_arith as GA
    f32 = np.float32
    return {
        "single_row": lambda t, b, x, N, K: GA.emulate_kq(t, b, np.asarray(x, f32), N, K).astype(f32),
        "batched": lambda t, b, x, N, K: GA.emulate(t, b, np.asarray(x, f32)[None], N, K)[0].astype(f32),
        "tensor_core": lambda t, b, x, N, K: TA.emulate_tc(t, b, np.asarray(x, f32)[None], N, K)[0].astype(f32),
    }


@pytest.mark.parametrize("n_layers", [2, 8, 32, 80])
def test_logits_at_depth(monkeypatch, oracle_mod, n_layers):
    import oracle.model_ref as MR
    from swq.model import LlamaConfig, rope_freqs
    from test_gpu_model import _weights
    cfg = LlamaConfig(n_layers=n_layers, dim=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024, vocab=1000,
                      max_seq=8)
    W = _weights(cfg, seed=21)
    ref = MR.RefLlama(cfg, W, rope_freqs(cfg), cfg.max_seq)
    want = [ref.forward(tok, p) for p, tok in enumerate(TOKS)]
    errs = {}
    for name, fn in _forms().items():
        monkeypatch.setattr(MR, "matmul", fn)
        m = MR.RefLlama(cfg, W, rope_freqs(cfg), cfg.max_seq)
        errs[name] = max(rel_l2(m.forward(tok, p), w) for (p, tok), w in zip(enumerate(TOKS), want))
    assert errs["single_row"] <= 1e-4 and errs["batched"] <= 1e-4, errs
    assert 1e-3 <= errs["tensor_core"] <= 5e-2, errs
