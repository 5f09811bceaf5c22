"""Tiny dense Llama models written as GGUF files, for the model-level parity
tests and their golden logits.

Each variant is fully determined by its spec (shapes, per-layer GGML types,
seeds), so the file is rebuilt byte for byte wherever the tests run and only
its SHA-256 and the reference's logits are stored (tests/golden/).

* "mix":  2 layers, hidden 256, 4 query / 2 kv heads of 64, FFN 512, vocab
          300; every one of the seven formats appears; the layers have
          different type mixes; F32 embedding table; Q6_K output matrix;
          general.alignment 64; no llama.vocab_size (the token list sets it).
* "tied": the same shape with a Q4_K_M-style mix on both layers, a Q8_0
          embedding table and no output.weight (the LM head is the
          embedding table, src/model.h:776-779), as small Llama models ship.
* "neox": the same shape under the "qwen2" architecture name (no biases),
          which the reference runs with neox RoPE, pairs (i, i + head_dim/2)
          (src/model.h:629-634).
* "bias": "qwen2" with q/k/v biases (src/model.h:291-294).
* "qknorm": "qwen3" with per-head q/k RMSNorm weights (src/model.h:296-318).
* "hybrid": "qwen35" (neox RoPE) whose layer 0 is a GatedDeltaNet layer
          (qwen35.attention.layer_types = [1, 0]; 2 key heads and 4 value
          heads of 32, conv width 4; attn_qkv, attn_gate, ssm_beta,
          ssm_alpha, ssm_dt, ssm_out projections, F32 ssm_a, ssm_conv1d,
          ssm_norm) and layer 1 full attention (src/model.h:369-513).  Its
          attn_qkv scales are small: the reference applies the delta rule to
          unnormalised keys, which diverges once beta |k|^2 > 2.
"""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

from swq import gguf as G
from swq import synth

TOKENS = [7, 123, 45, 299, 0, 200]   # teacher-forced tokens at positions 0..5

SHAPE = dict(layers=2, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=300, context=32)
# GatedDeltaNet layers of the "hybrid" variant
LINEAR = dict(n_k=2, n_v=4, k_hd=32, v_hd=32, conv=4)
_STEMS = {"wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output", "w_gate": "ffn_gate",
          "w_up": "ffn_up", "w_down": "ffn_down"}

VARIANTS = {
    "mix": dict(
        alignment=64, embd=G.F32, output=G.Q6_K, vocab_key=False,
        layers=[dict(wq=G.Q4_K, wk=G.Q4_K, wv=G.Q6_K, wo=G.Q4_0, w_gate=G.Q4_K, w_up=G.Q4_K, w_down=G.Q6_K),
                dict(wq=G.Q5_K, wk=G.Q5_K, wv=G.Q8_0, wo=G.Q2_K, w_gate=G.Q3_K, w_up=G.Q3_K, w_down=G.Q4_K)]),
    "tied": dict(
        alignment=32, embd=G.Q8_0, output=None, vocab_key=True,
        layers=[dict(wq=G.Q4_K, wk=G.Q4_K, wv=G.Q6_K, wo=G.Q4_K, w_gate=G.Q4_K, w_up=G.Q4_K, w_down=G.Q6_K)] * 2),
    "neox": dict(
        arch="qwen2", alignment=32, embd=G.F32, output=G.Q6_K, vocab_key=True,
        layers=[dict(wq=G.Q4_K, wk=G.Q4_K, wv=G.Q6_K, wo=G.Q4_K, w_gate=G.Q4_K, w_up=G.Q4_K, w_down=G.Q6_K)] * 2),
    "bias": dict(
        arch="qwen2", alignment=32, embd=G.F32, output=G.Q6_K, vocab_key=True, biases=True,
        layers=[dict(wq=G.Q4_K, wk=G.Q4_K, wv=G.Q6_K, wo=G.Q4_K, w_gate=G.Q4_K, w_up=G.Q4_K, w_down=G.Q6_K)] * 2),
    "qknorm": dict(
        arch="qwen3", alignment=32, embd=G.F32, output=G.Q6_K, vocab_key=True, qk_norm=True,
        layers=[dict(wq=G.Q4_K, wk=G.Q4_K, wv=G.Q6_K, wo=G.Q4_K, w_gate=G.Q4_K, w_up=G.Q4_K, w_down=G.Q6_K)] * 2),
    "hybrid": dict(
        arch="qwen35", alignment=32, embd=G.F32, output=G.Q6_K, vocab_key=True, linear=(0,),
        layers=[dict(w_qkv=G.Q4_K, w_z=G.Q8_0, w_beta=G.Q8_0, w_alpha=G.Q8_0, w_dt=G.Q8_0, w_ssm_out=G.Q8_0,
                     w_gate=G.Q4_K, w_up=G.Q4_K, w_down=G.Q6_K),
                dict(wq=G.Q4_K, wk=G.Q4_K, wv=G.Q6_K, wo=G.Q4_K, w_gate=G.Q4_K, w_up=G.Q4_K, w_down=G.Q6_K)]),
}
_LINEAR_STEMS = {"w_qkv": "attn_qkv", "w_z": "attn_gate", "w_beta": "ssm_beta", "w_alpha": "ssm_alpha",
                 "w_dt": "ssm_dt", "w_ssm_out": "ssm_out"}


def _shapes(s):
    hd = s["hidden"] // s["heads"]
    q, kv = s["heads"] * hd, s["kv_heads"] * hd
    return {"wq": (q, s["hidden"]), "wk": (kv, s["hidden"]), "wv": (kv, s["hidden"]), "wo": (s["hidden"], q),
            "w_gate": (s["ffn"], s["hidden"]), "w_up": (s["ffn"], s["hidden"]), "w_down": (s["hidden"], s["ffn"])}


def _linear_shapes(s):
    L = LINEAR
    key, val = L["n_k"] * L["k_hd"], L["n_v"] * L["v_hd"]
    return {"w_qkv": (2 * key + val, s["hidden"]), "w_z": (val, s["hidden"]), "w_beta": (L["n_v"], s["hidden"]),
            "w_alpha": (L["n_v"], s["hidden"]), "w_dt": (L["n_v"], s["hidden"]), "w_ssm_out": (s["hidden"], val),
            "w_gate": (s["ffn"], s["hidden"]), "w_up": (s["ffn"], s["hidden"]), "w_down": (s["hidden"], s["ffn"])}


def write(path: Path, variant: str) -> Path:
    """Write the variant's GGUF file at path."""
    v, s = VARIANTS[variant], SHAPE
    a = v.get("arch", "llama")
    rng = np.random.default_rng({"mix": 11, "tied": 12, "neox": 13, "bias": 14, "qknorm": 15,
                                 "hybrid": 16}[variant])
    meta = {
        "general.architecture": a,
        "general.name": f"tiny-{variant}",
        "general.alignment": v["alignment"],
        f"{a}.context_length": s["context"],
        f"{a}.embedding_length": s["hidden"],
        f"{a}.block_count": s["layers"],
        f"{a}.feed_forward_length": s["ffn"],
        f"{a}.attention.head_count": s["heads"],
        f"{a}.attention.head_count_kv": s["kv_heads"],
        f"{a}.rope.freq_base": G.GGUFValue(G.FLOAT32, 500000.0),
        f"{a}.attention.layer_norm_rms_epsilon": G.GGUFValue(G.FLOAT32, 1e-5),
        "tokenizer.ggml.model": "llama",
        "tokenizer.ggml.tokens": [f"<t{i}>" for i in range(s["vocab"])],
        "tokenizer.ggml.scores": [float(-i) for i in range(s["vocab"])],
    }
    if v["vocab_key"]:
        meta[f"{a}.vocab_size"] = s["vocab"]
    linear = v.get("linear", ())
    if linear:
        meta[f"{a}.attention.layer_types"] = [1 if li in linear else 0 for li in range(s["layers"])]
        meta[f"{a}.attention.linear_key_length"] = LINEAR["k_hd"]
        meta[f"{a}.attention.linear_value_length"] = LINEAR["v_hd"]
        meta[f"{a}.attention.linear_head_count_kv"] = LINEAR["n_k"]
        meta[f"{a}.attention.linear_head_count"] = LINEAR["n_v"]
        meta[f"{a}.ssm.conv_kernel"] = LINEAR["conv"]
    tensors = []

    def norm(name):
        tensors.append((name, G.F32, (s["hidden"],), (1 + 0.01 * rng.standard_normal(s["hidden"])).astype(np.float32)))

    def mat(name, t, N, K, seed, scale=1.0):
        tensors.append((name, t, (K, N), synth.random_blocks(t, N, K, seed=seed, d_scale=2e-3 * scale,
                                                             dmin_scale=1e-3 * scale)))

    if v["embd"] == G.F32:
        tensors.append(("token_embd.weight", G.F32, (s["hidden"], s["vocab"]),
                        rng.standard_normal((s["vocab"], s["hidden"])).astype(np.float32)))
    else:
        mat("token_embd.weight", v["embd"], s["vocab"], s["hidden"], 900)
    norm("output_norm.weight")
    if v["output"] is not None:
        mat("output.weight", v["output"], s["vocab"], s["hidden"], 901)
    for li, lt in enumerate(v["layers"]):
        norm(f"blk.{li}.attn_norm.weight")
        norm(f"blk.{li}.ffn_norm.weight")
        if li in linear:
            for j, (key, (N, K)) in enumerate(_linear_shapes(s).items()):
                stem = _LINEAR_STEMS.get(key) or _STEMS[key]
                # q/k/v small enough that the delta rule, which the reference
                # runs on unnormalised keys, stays stable (beta |k|^2 < 2)
                mat(f"blk.{li}.{stem}.weight", lt[key], N, K, 1000 + 10 * li + j,
                    scale=0.0075 if key == "w_qkv" else 1.0)
            nv, val, cw = LINEAR["n_v"], LINEAR["n_v"] * LINEAR["v_hd"], LINEAR["conv"]
            tensors.append((f"blk.{li}.ssm_a", G.F32, (nv,), (0.5 * rng.standard_normal(nv)).astype(np.float32)))
            tensors.append((f"blk.{li}.ssm_conv1d.weight", G.F32, (cw, val),
                            (0.5 * rng.standard_normal((val, cw))).astype(np.float32)))
            tensors.append((f"blk.{li}.ssm_norm.weight", G.F32, (val,),
                            (1 + 0.1 * rng.standard_normal(val)).astype(np.float32)))
            continue
        for j, (key, (N, K)) in enumerate(_shapes(s).items()):
            mat(f"blk.{li}.{_STEMS[key]}.weight", lt[key], N, K, 1000 + 10 * li + j)
        hd = s["hidden"] // s["heads"]
        if v.get("biases"):
            for stem, n in (("attn_q", s["heads"] * hd), ("attn_k", s["kv_heads"] * hd), ("attn_v", s["kv_heads"] * hd)):
                tensors.append((f"blk.{li}.{stem}.bias", G.F32, (n,), rng.standard_normal(n).astype(np.float32)))
        if v.get("qk_norm"):
            for stem in ("attn_q_norm", "attn_k_norm"):
                tensors.append((f"blk.{li}.{stem}.weight", G.F32, (hd,),
                                (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)))
    G.write_gguf(path, meta, tensors, alignment=v["alignment"])
    return path


def sha256(path: Path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()
