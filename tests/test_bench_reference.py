"""bench.py's reference decode leg on the CPU: a GGUF file of a dense Llama
shape written by the bench, loaded and run by the reference's own Model
(src/model.h compiled from source), at a tiny shape."""
import sys

import numpy as np
import pytest

from conftest import REPO

if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def _tiny():
    from swq.model import LlamaConfig
    return LlamaConfig(n_layers=2, dim=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=512, vocab=300, max_seq=32)


def test_bench_model_file_reads_back(tmp_path):
    import bench
    from swq import gguf as G
    cfg = _tiny()
    size = bench.write_llama_gguf(tmp_path / "m.gguf", cfg)
    g = G.GGUFFile(tmp_path / "m.gguf")
    assert size == g.file_size
    got = G.llama_config(g)
    for k in ("n_layers", "dim", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "max_seq", "types"):
        assert getattr(got, k) == getattr(cfg, k), k
    assert np.float32(got.theta) == np.float32(cfg.theta) and np.float32(got.eps) == np.float32(cfg.eps)
    assert g.tensors["token_embd.weight"].type == G.Q4_K


def test_reference_decode_timing_runs(tmp_path):
    from oracle.ref_model import model_ref_available
    if not model_ref_available():
        pytest.skip("reference model library not built (needs the reference sources)")
    import bench
    r = bench.ref_decode_timing(_tiny(), seconds=1.0, max_tokens=3, workdir=str(tmp_path))
    assert r["finite_logits"] and r["tok_s"] > 0 and r["kind"] == "reference"
    assert "3 Model::forward calls" in r["sample"]
    assert list(tmp_path.iterdir()) == []  # the model file is gone


def test_cpu_gemv_timing_threads():
    """At least min_steps steps of per_step GEMVs and at least `seconds`,
    after the warm-up GEMVs; the steps that ran are reported."""
    import bench
    r = bench.cpu_gemv_timing(seconds=0.05, min_steps=3, copies=2, threads=1, warmup=2, per_step=2)
    assert r["cores"] == 1 and r["value"] > 0 and "1 OpenMP threads" in r["sample"]
    assert r["steps"] >= 3 and r["gemvs"] == 2 * r["steps"] and r["seconds"] >= 0.05
    assert "after 2 warm-up GEMVs" in r["sample"]
    assert isinstance(bench.cpu_model(), str)


def test_decode_context_synthetic_is_the_kv_fill(monkeypatch):
    """The synthetic decode context (--decode-context synthetic): the same
    tokens and random K/V fill as the decode measurements used before the
    prefill context became the default."""
    import bench
    assert bench.DECODE_CONTEXT == "prefill"
    monkeypatch.setattr(bench, "DECODE_CONTEXT", "synthetic")

    class Dec:
        rows = 3
        cfg = type("Cfg", (), {"vocab": 1000})()

        def reset(self, tokens, pos):
            self.reset_args = (list(tokens), pos)

        def fill_kv(self, n):
            self.filled = n

    d = Dec()
    out = bench._build_context(d, 512, seed=1)
    assert d.reset_args == ([1, 8, 15], 0) and d.filled == 512
    assert out == {"context": "synthetic K/V for 512 positions"}
