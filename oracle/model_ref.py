"""CPU restatement of the reference's dense Llama decode forward
(TEST INFRASTRUCTURE ONLY).

``RefLlama.forward(token, pos)`` follows Model::forward (src/model.h:257-543)
on the full-attention, dense-FFN path, in fp32 numpy:

  x = token_embd[token]                                   (:265)
  per layer: xb = rmsnorm(x, attn_norm)                   (:272, src/tensor.h:1028-1033)
             q, k, v = W{q,k,v} . xb                       (:284-289)
             + biases, per-head q/k RMSNorm when present   (:291-318)
             rope(q, k) at pos, interleaved pairs          (:322-323, src/tensor.h:1068-1107)
               (pairs (i, i + head_dim/2) for the neox architectures, :1121-1161)
             cache k, v at pos                             (:326-327)
             per head: scores = q.k_t / sqrt(head_dim), t <= pos; softmax; out = sum p v_t
                                                           (:329-361, src/tensor.h:1036-1047)
             x += Wo . out                                 (:363-366)
             xb = rmsnorm(x, ffn_norm); h = silu(Wg . xb) * (Wu . xb); x += Wd . h
                                                           (:521-541, src/tensor.h:1050-1064)
  logits = Woutput . rmsnorm(x, output_norm)               (:545-551)

The quantized matmuls are the reference's own routine compiled from source
(oracle/_ref) when it was built, else this package's C restatement in the
reference's accumulation order.  Per-layer type mixes (cfg.layer_type_map) and
an embedding table given as (GGML type, blocks) are read as the reference's
Model::load reads them.  Only tests use this module.

Pinned: tests/test_gguf.py runs it against the reference's own Model::forward
(src/model.h compiled from source, oracle/model_shim.cpp) on tiny GGUF models,
live and through the golden logits the reference produced
(tests/golden/golden_llama_*.npz); they agree to ~4e-7 relative L2.
"""
from __future__ import annotations

import numpy as np

from . import gemv as _port_gemv
from . import ref_available, ref_gemv

F32 = np.float32


def matmul(type_id: int, blocks: np.ndarray, x: np.ndarray, N: int, K: int) -> np.ndarray:
    if ref_available():
        return ref_gemv(type_id, blocks, x, N, K)
    return _port_gemv(type_id, blocks, x, N, K, format_order=False)


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    ss = F32(0.0)
    for v in x.astype(F32):  # sequential fp32 sum, as the reference loop
        ss = F32(ss + v * v)
    scale = F32(1.0) / np.sqrt(F32(ss / F32(len(x)) + F32(eps)))
    return (x * scale * w).astype(F32)


def rope_interleaved(vec: np.ndarray, head_dim: int, pos: int, freqs: np.ndarray) -> np.ndarray:
    out = vec.astype(F32).copy()
    heads = len(vec) // head_dim
    for h in range(heads):
        for i in range(0, head_dim, 2):
            angle = F32(pos) * freqs[i // 2]
            c, s = np.cos(angle, dtype=F32), np.sin(angle, dtype=F32)
            a, b = out[h * head_dim + i], out[h * head_dim + i + 1]
            out[h * head_dim + i] = a * c - b * s
            out[h * head_dim + i + 1] = a * s + b * c
    return out


def rope_neox(vec: np.ndarray, head_dim: int, pos: int, freqs: np.ndarray) -> np.ndarray:
    """Pairs (i, i + head_dim/2) (cpu_rope_neox_apply, src/tensor.h:1121-1161)."""
    out = vec.astype(F32).copy()
    half = head_dim // 2
    for h in range(len(vec) // head_dim):
        for i in range(half):
            angle = F32(pos) * freqs[i]
            c, s = np.cos(angle, dtype=F32), np.sin(angle, dtype=F32)
            a, b = out[h * head_dim + i], out[h * head_dim + i + half]
            out[h * head_dim + i] = a * c - b * s
            out[h * head_dim + i + half] = b * c + a * s
    return out


def sigmoid(x) -> np.float32:
    with np.errstate(over="ignore"):
        return F32(F32(1.0) / (F32(1.0) + np.exp(F32(-x), dtype=F32)))


def gdn_step(qkv, z, beta, alpha, dt, ssm_a, conv_w, norm_w, S, conv, n_k, n_v, k_hd, v_hd, cw):
    """One GatedDeltaNet step after the projections, the loops of
    src/model.h:421-504 in fp32 (one row; S [n_v, k_hd, v_hd] and conv
    [value_dim, cw] updated in place).  z, beta, alpha, dt, ssm_a, conv_w,
    norm_w may be None, as the reference's missing tensors."""
    key_dim, value_dim = n_k * k_hd, n_v * v_hd
    q, k, v = qkv[:key_dim], qkv[key_dim:2 * key_dim], qkv[2 * key_dim:2 * key_dim + value_dim].astype(F32)
    if conv_w is not None and cw > 0:
        conv[:, :cw - 1] = conv[:, 1:].copy()
        conv[:, cw - 1] = v
        out = np.zeros(value_dim, F32)
        for w in range(cw):  # sequential sum over the taps, channel by channel
            out = (out + (conv_w[:, w] * conv[:, w]).astype(F32)).astype(F32)
        v = out
    y = np.zeros(value_dim, F32)
    for h in range(n_v):
        kh = h % n_k
        qh, khv = q[kh * k_hd:(kh + 1) * k_hd].astype(F32), k[kh * k_hd:(kh + 1) * k_hd].astype(F32)
        vh = v[h * v_hd:(h + 1) * v_hd]
        base = np.exp(F32(ssm_a[h]), dtype=F32) if ssm_a is not None else F32(1.0)
        ag = sigmoid(alpha[h]) if alpha is not None else F32(1.0)
        log_decay = F32(-base * ag)
        if dt is not None:
            log_decay = F32(log_decay * sigmoid(dt[h]))
        decay = np.exp(log_decay, dtype=F32)
        b = sigmoid(beta[h]) if beta is not None else F32(1.0)
        Sh = S[h]
        pred = np.zeros(v_hd, F32)
        for i in range(k_hd):  # sum over i in order, as the reference's loop
            pred = (pred + (Sh[i] * khv[i]).astype(F32)).astype(F32)
        delta = (vh - pred).astype(F32)
        for i in range(k_hd):
            Sh[i] = ((decay * Sh[i]).astype(F32) + ((b * khv[i]).astype(F32) * delta).astype(F32)).astype(F32)
        yh = np.zeros(v_hd, F32)
        for i in range(k_hd):
            yh = (yh + (Sh[i] * qh[i]).astype(F32)).astype(F32)
        if norm_w is not None:
            ss = F32(0.0)
            for val in yh:
                ss = F32(ss + val * val)
            ss = F32(1.0) / np.sqrt(F32(ss / F32(v_hd) + F32(1e-5)))
            yh = (yh * ss * norm_w[h * v_hd:(h + 1) * v_hd]).astype(F32)
        y[h * v_hd:(h + 1) * v_hd] = yh
    zz = z if z is not None else np.zeros(value_dim, F32)
    return np.array([F32(y[d] * sigmoid(zz[d])) for d in range(value_dim)], F32)


def softmax(x: np.ndarray) -> np.ndarray:
    m = x.max()
    e = np.exp((x - m).astype(F32)).astype(F32)
    return (e / e.sum(dtype=F32)).astype(F32)


class RefLlama:
    """cfg: swq.model.LlamaConfig-like (n_layers, dim, n_heads, n_kv_heads,
    head_dim, ffn, vocab, eps, types); weights: the host arrays LlamaDecoder takes."""

    def __init__(self, cfg, weights: dict, freqs: np.ndarray, max_seq: int):
        te = weights["token_embd"]
        if isinstance(te, tuple):  # (GGML type, blocks): dequantized at load, src/model.h:771-772
            from . import dequantize as _port_dequant
            from . import ref_dequantize
            deq = ref_dequantize if ref_available() else _port_dequant
            weights = dict(weights, token_embd=deq(te[0], np.asarray(te[1]), cfg.vocab * cfg.dim).reshape(
                cfg.vocab, cfg.dim))
        self.cfg, self.W, self.freqs = cfg, weights, freqs.astype(F32)
        self.kc = np.zeros((cfg.n_layers, max_seq, cfg.n_kv_heads * cfg.head_dim), F32)
        self.vc = np.zeros_like(self.kc)
        lin = getattr(cfg, "linear_layers", ())
        if lin:  # GatedDeltaNet state per linear layer (LinearAttentionState, src/model.h:131-166)
            self.S = np.zeros((len(lin), cfg.lin_n_v, cfg.lin_k_hd, cfg.lin_v_hd), F32)
            self.conv = np.zeros((len(lin), cfg.lin_value_dim, max(1, cfg.lin_conv)), F32)

    def forward(self, token: int, pos: int) -> np.ndarray:
        c, W = self.cfg, self.W
        hd, nh, nkv = c.head_dim, c.n_heads, c.n_kv_heads
        q_dim, kv_dim = nh * hd, nkv * hd
        x = np.asarray(W["token_embd"][token], F32).copy()
        for li, L in enumerate(W["layers"]):
            t = c.layer_type_map(li) if hasattr(c, "layer_type_map") else c.types
            xb = rmsnorm(x, L["attn_norm"], c.eps)
            if li in getattr(c, "linear_layers", ()):
                x = (x + self._gdn(li, L, t, xb)).astype(F32)
                x = self._ffn(L, t, x)
                continue
            q = matmul(t["wq"], L["wq"], xb, q_dim, c.dim)
            k = matmul(t["wk"], L["wk"], xb, kv_dim, c.dim)
            v = matmul(t["wv"], L["wv"], xb, kv_dim, c.dim)
            # optional biases, then per-head RMSNorm of q and k (src/model.h:291-318)
            q = (q + L["bq"]).astype(F32) if "bq" in L else q
            k = (k + L["bk"]).astype(F32) if "bk" in L else k
            v = (v + L["bv"]).astype(F32) if "bv" in L else v
            if "q_norm" in L:
                q = np.concatenate([rmsnorm(q[h * hd:(h + 1) * hd], L["q_norm"], c.eps) for h in range(nh)])
            if "k_norm" in L:
                k = np.concatenate([rmsnorm(k[h * hd:(h + 1) * hd], L["k_norm"], c.eps) for h in range(nkv)])
            rope = rope_neox if getattr(c, "rope_neox", False) else rope_interleaved
            q = rope(q, hd, pos, self.freqs)
            k = rope(k, hd, pos, self.freqs)
            self.kc[li, pos], self.vc[li, pos] = k, v
            att = np.zeros(q_dim, F32)
            mul = nh // nkv
            for h in range(nh):
                kvh = h // mul
                qh = q[h * hd:(h + 1) * hd]
                ks = self.kc[li, :pos + 1, kvh * hd:(kvh + 1) * hd]
                vs = self.vc[li, :pos + 1, kvh * hd:(kvh + 1) * hd]
                p = softmax((ks @ qh).astype(F32) / np.sqrt(F32(hd)))
                att[h * hd:(h + 1) * hd] = (p @ vs).astype(F32)
            x = (x + matmul(t["wo"], L["wo"], att, c.dim, q_dim)).astype(F32)
            x = self._ffn(L, t, x)
        x = rmsnorm(x, W["output_norm"], c.eps)
        return matmul(c.types["output"], W["output"], x, c.vocab, c.dim)

    def _ffn(self, L, t, x):
        """x + FFN(rmsnorm(x, ffn_norm)): dense SwiGLU (src/model.h:519-541) or MoE."""
        c = self.cfg
        xb = rmsnorm(x, L["ffn_norm"], c.eps)
        if "router" in L:
            return (x + self._moe(L, t, xb)).astype(F32)
        g = matmul(t["w_gate"], L["w_gate"], xb, c.ffn, c.dim)
        u = matmul(t["w_up"], L["w_up"], xb, c.ffn, c.dim)
        with np.errstate(over="ignore"):  # exp(-g) = inf for very negative g: silu -> -0, as expf
            hmid = (g / (F32(1.0) + np.exp(-g)) * u).astype(F32)
        return (x + matmul(t["w_down"], L["w_down"], hmid, c.dim, c.ffn)).astype(F32)

    def _gdn(self, li, L, t, xb):
        """A GatedDeltaNet layer's output projection input and output
        (src/model.h:369-513): projections of xb, gdn_step, ssm_out."""
        c = self.cfg
        kd, vd, nv, H = c.lin_key_dim, c.lin_value_dim, c.lin_n_v, c.dim
        qkv = matmul(t["w_qkv"], L["w_qkv"], xb, 2 * kd + vd, H)
        proj = {k: matmul(t[k], L[k], xb, n, H) if k in L else None
                for k, n in (("w_z", vd), ("w_beta", nv), ("w_alpha", nv), ("w_dt", nv))}
        j = c.linear_layers.index(li)
        conv = L.get("conv1d")
        y = gdn_step(qkv, proj["w_z"], proj["w_beta"], proj["w_alpha"], proj["w_dt"], L.get("ssm_a"),
                     None if conv is None else np.asarray(conv, F32).reshape(vd, c.lin_conv), L.get("ssm_norm"),
                     self.S[j], self.conv[j], c.lin_n_k, nv, c.lin_k_hd, c.lin_v_hd, c.lin_conv)
        return matmul(t["w_ssm_out"], L["w_ssm_out"], y, H, vd)

    def _swiglu(self, tg, gb, tu, ub, td, db, xb, f):
        c = self.cfg
        g = matmul(tg, gb, xb, f, c.dim)
        u = matmul(tu, ub, xb, f, c.dim)
        with np.errstate(over="ignore"):
            h = (g / (F32(1.0) + np.exp(-g)) * u).astype(F32)
        return matmul(td, db, h, c.dim, f)

    def _moe(self, L, t, xb):
        """MoE FFN (no counterpart in the reference, whose FFN is dense): fp32
        router logits, the top_k experts with softmax weights over their
        logits (oracle/moe_oracle.c), each a SwiGLU FFN, summed in slot order
        onto the shared expert's output."""
        from . import moe_router_logits, moe_topk_softmax
        c = self.cfg
        E, F, Fs = c.n_experts, c.expert_ffn, c.shared_ffn
        logits = moe_router_logits(L["router"], xb[None]).astype(F32)
        ids, w = moe_topk_softmax(logits, c.top_k)
        self.last_ids = ids[0]
        y = np.zeros(c.dim, F32)
        if Fs:
            y = self._swiglu(t["w_gate_shexp"], L["w_gate_shexp"], t["w_up_shexp"], L["w_up_shexp"],
                             t["w_down_shexp"], L["w_down_shexp"], xb, Fs).astype(F32)
        parts = {nm: np.asarray(L[nm]).reshape(E, -1) for nm in ("w_gate_exps", "w_up_exps", "w_down_exps")}
        for j in range(c.top_k):
            e = int(ids[0, j])
            out = self._swiglu(t["w_gate_exps"], parts["w_gate_exps"][e], t["w_up_exps"], parts["w_up_exps"][e],
                               t["w_down_exps"], parts["w_down_exps"][e], xb, F)
            y = (y + w[0, j] * out).astype(F32)
        return y
