"""Device-resident Llama decode around the quantized GEMVs.

`LlamaDecoder` runs the reference's decode forward (Model::forward,
src/model.h:257-543, dense Llama path) entirely on one GPU through libswq:
embedding row, per layer RMSNorm, q/k/v GEMVs, RoPE + KV-cache append,
grouped-query attention, o GEMV, residual, RMSNorm, gate+up GEMV, SiLU-mul,
down GEMV, residual; final RMSNorm, LM-head GEMV and greedy argmax.  Matrices
of one type that read the same input are stacked into one GEMV (q with k,
gate with up), and every residual add runs in one kernel with the RMSNorm
after it.  `rows` sequences
decode in step.  The position lives in device memory, so one decode step is
captured once in a CUDA graph and replayed per token.

Weights are GGUF blocks in device memory: either given (host arrays, for the
tests) or synthetic -- seeded random blocks with the benchmark's value
distributions, generated on the device -- in the Q4_K_M mix (Q6_K for attn_v,
ffn_down and the output matrix, Q4_K elsewhere).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import lib as _lib_mod  # noqa: F401  (module import for the ctypes table)
from .lib import (GEMM_NOALLOC_MAX_X_ELEMS, OPT_TENSOR_CORE_MIN_M, add_rmsnorm, argmax, attention_decode,
                  attention_workspace_bytes, decode_advance, embed, gemm, gemm_noalloc, get_option, rmsnorm,
                  rope_kv, silu_mul)
from .synth import LAYOUT, Q4_K, Q6_K, Q8_0, row_bytes


@dataclass
class LlamaConfig:
    n_layers: int = 32
    dim: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    eps: float = 1e-5
    theta: float = 5e5
    rope_neox: bool = False          # Llama: interleaved pairs
    max_seq: int = 1024
    # GGML types of the Q4_K_M mix
    types: dict = field(default_factory=lambda: {"wq": Q4_K, "wk": Q4_K, "wv": Q6_K, "wo": Q4_K,
                                                 "w_gate": Q4_K, "w_up": Q4_K, "w_down": Q6_K, "output": Q6_K})

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def shapes(self) -> dict:
        """name -> (N rows, K columns) of every quantized matrix of a layer."""
        return {"wq": (self.q_dim, self.dim), "wk": (self.kv_dim, self.dim), "wv": (self.kv_dim, self.dim),
                "wo": (self.dim, self.q_dim), "w_gate": (self.ffn, self.dim), "w_up": (self.ffn, self.dim),
                "w_down": (self.dim, self.ffn)}

    def weight_bytes_per_token(self) -> int:
        """Quantized weight bytes one decode step reads (all layers + LM head)."""
        per_layer = sum(n * row_bytes(self.types[k], kk) for k, (n, kk) in self.shapes().items())
        return self.n_layers * per_layer + self.vocab * row_bytes(self.types["output"], self.dim)


def rope_freqs(cfg: LlamaConfig) -> np.ndarray:
    """freqs[i] = 1 / theta^(2i / rope_dim) (src/model.h:903-907), fp32."""
    i = np.arange(cfg.head_dim // 2, dtype=np.float32)
    return (1.0 / np.power(np.float32(cfg.theta), (2.0 * i) / np.float32(cfg.head_dim))).astype(np.float32)


def synthetic_blocks(type_id: int, N: int, K: int, generator, device):
    """Seeded random GGUF blocks on the device: random bytes, then d = fp16(|N(0,1)|
    * 2e-3) and dmin = fp16(|N(0,1)| * 1e-3) written into every block (Q8_0
    quants kept in -127..127)."""
    import torch
    qk, bb, d_off, m_off = LAYOUT[type_id]
    nb = K // qk
    b = torch.randint(0, 256, (N, nb, bb), dtype=torch.uint8, device=device, generator=generator)
    d = (torch.randn((N, nb), device=device, generator=generator).abs() * 2e-3).half()
    b[:, :, d_off:d_off + 2] = d.view(torch.uint8).view(N, nb, 2)
    if m_off is not None:
        m = (torch.randn((N, nb), device=device, generator=generator).abs() * 1e-3).half()
        b[:, :, m_off:m_off + 2] = m.view(torch.uint8).view(N, nb, 2)
    if type_id == Q8_0:
        q = b[:, :, 2:]
        q[q == 0x80] = 0x81
    return b.reshape(-1)


class LlamaDecoder:
    def __init__(self, cfg: LlamaConfig, rows: int = 1, device="cuda", seed: int = 0, weights: dict | None = None,
                 max_steps: int = 4096):
        """weights: None for synthetic weights, else host arrays: 'token_embd'
        [vocab, dim] fp32, 'output_norm' [dim], 'output' blocks, and per layer
        'layers'[l] with 'attn_norm', 'ffn_norm' [dim] fp32 and the blocks of
        wq wk wv wo w_gate w_up w_down."""
        import torch
        self.cfg, self.rows, self.device = cfg, rows, torch.device(device)
        dev = self.device
        t = cfg.types
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        f32 = dict(dtype=torch.float32, device=dev)

        def blocks(name, N, K, host):
            if host is not None:
                return torch.from_numpy(np.ascontiguousarray(host).reshape(-1)).to(dev)
            return synthetic_blocks(t[name], N, K, g, dev)

        W = weights or {}
        self.token_embd = (torch.from_numpy(np.asarray(W["token_embd"], np.float32)).to(dev) if weights
                           else torch.randn((cfg.vocab, cfg.dim), generator=g, **f32))
        self.output_norm = (torch.from_numpy(np.asarray(W["output_norm"], np.float32)).to(dev) if weights
                            else 1.0 + 0.01 * torch.randn(cfg.dim, generator=g, **f32))
        self.output = blocks("output", cfg.vocab, cfg.dim, W.get("output"))
        self.fuse_gate_up = t["w_gate"] == t["w_up"]
        self.fuse_qk = t["wq"] == t["wk"]
        self.layers = []
        for layer in range(cfg.n_layers):
            lw = W["layers"][layer] if weights else {}
            L = {}
            for name in ("attn_norm", "ffn_norm"):
                L[name] = (torch.from_numpy(np.asarray(lw[name], np.float32)).to(dev) if weights
                           else 1.0 + 0.01 * torch.randn(cfg.dim, generator=g, **f32))
            for name, (N, K) in cfg.shapes().items():
                L[name] = blocks(name, N, K, lw.get(name))
            if self.fuse_gate_up:  # rows of gate then rows of up: one GEMV
                L["w_gate_up"] = torch.cat([L.pop("w_gate"), L.pop("w_up")])
            if self.fuse_qk:  # rows of q then rows of k
                L["w_qk"] = torch.cat([L.pop("wq"), L.pop("wk")])
            self.layers.append(L)
        self.freqs = torch.from_numpy(rope_freqs(cfg)).to(dev)
        B = rows
        self.x = torch.zeros((B, cfg.dim), **f32)
        self.xb = torch.zeros_like(self.x)
        self.qk = torch.zeros((B, cfg.q_dim + cfg.kv_dim), **f32)  # q then k, per row
        self.v = torch.zeros((B, cfg.kv_dim), **f32)
        self.att = torch.zeros((B, cfg.q_dim), **f32)
        self.gu = torch.zeros((B, 2 * cfg.ffn), **f32)
        self.h = torch.zeros((B, cfg.ffn), **f32)
        self.logits = torch.zeros((B, cfg.vocab), **f32)
        self.kcache = torch.zeros((cfg.n_layers, B, cfg.max_seq, cfg.kv_dim), **f32)
        self.vcache = torch.zeros_like(self.kcache)
        self.tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.step_no = torch.zeros(1, dtype=torch.int32, device=dev)
        self.history = torch.zeros((max_steps, B), dtype=torch.int32, device=dev)
        self.ws_bytes = attention_workspace_bytes(cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, B, cfg.max_seq)
        self.ws = torch.zeros(max(1, self.ws_bytes // 4), **f32)  # zero-filled, as the kernel expects
        self.max_steps = max_steps
        self.steps_issued = 0
        self.stream = torch.cuda.Stream(device=dev)
        self.graph = None

    # ------------------------------------------------------------ one token
    def _gemm(self, type_id, W, X, Y, M, N, K, stream):
        # Rows that take the tensor-core GEMM use its allocation-free form, so
        # a captured step holds no allocation (one stream orders the calls).
        if M >= get_option(OPT_TENSOR_CORE_MIN_M) and M * K <= GEMM_NOALLOC_MAX_X_ELEMS:
            gemm_noalloc(type_id, W, X, Y, M, N, K, stream=stream)
        else:
            gemm(type_id, W, X, Y, M, N, K, stream=stream)

    def step(self, greedy: bool = True) -> None:
        """One decode step for all rows at position *pos: logits of the current
        tokens; with greedy, tokens <- argmax (also into history) and pos += 1."""
        c, B, s = self.cfg, self.rows, self.stream
        t = c.types
        gemm = self._gemm  # noqa: F811
        ld = c.q_dim + c.kv_dim
        q, k = self.qk, self.qk[:, c.q_dim:]
        embed(self.x, self.token_embd, self.tokens, c.dim, c.vocab, B, stream=s)
        rmsnorm(self.xb, self.x, self.layers[0]["attn_norm"], c.dim, c.eps, B, stream=s)
        for li, L in enumerate(self.layers):
            if self.fuse_qk:
                gemm(t["wq"], L["w_qk"], self.xb, self.qk, B, ld, c.dim, stream=s)
            else:
                gemm(t["wq"], L["wq"], self.xb, self.att, B, c.q_dim, c.dim, stream=s)
                q[:, :c.q_dim].copy_(self.att)
                gemm(t["wk"], L["wk"], self.xb, self.v, B, c.kv_dim, c.dim, stream=s)
                k.copy_(self.v)
            gemm(t["wv"], L["wv"], self.xb, self.v, B, c.kv_dim, c.dim, stream=s)
            kc, vc = self.kcache[li], self.vcache[li]
            rope_kv(q, k, self.v, kc, vc, self.pos, self.freqs, c.q_dim, c.kv_dim, c.head_dim, c.head_dim,
                    c.rope_neox, B, c.max_seq, ldq=ld, ldk=ld, stream=s)
            attention_decode(self.att, q, kc, vc, self.pos, self.ws, self.ws_bytes, c.n_heads, c.n_kv_heads,
                             c.head_dim, B, c.max_seq, ldq=ld, stream=s)
            gemm(t["wo"], L["wo"], self.att, self.xb, B, c.dim, c.q_dim, stream=s)
            add_rmsnorm(self.xb, self.x, self.xb, L["ffn_norm"], c.dim, c.eps, B, stream=s)  # x += o; xb = norm(x)
            if self.fuse_gate_up:
                gemm(t["w_gate"], L["w_gate_up"], self.xb, self.gu, B, 2 * c.ffn, c.dim, stream=s)
            else:
                gemm(t["w_gate"], L["w_gate"], self.xb, self.h, B, c.ffn, c.dim, stream=s)
                self.gu[:, :c.ffn].copy_(self.h)
                gemm(t["w_up"], L["w_up"], self.xb, self.h, B, c.ffn, c.dim, stream=s)
                self.gu[:, c.ffn:].copy_(self.h)
            silu_mul(self.h, self.gu, self.gu[:, c.ffn:], c.ffn, B, 2 * c.ffn, stream=s)
            gemm(t["w_down"], L["w_down"], self.h, self.xb, B, c.dim, c.ffn, stream=s)
            if li + 1 < len(self.layers):  # x += down; xb = next layer's attention norm of x
                add_rmsnorm(self.xb, self.x, self.xb, self.layers[li + 1]["attn_norm"], c.dim, c.eps, B, stream=s)
            else:  # x += down; x = output norm of x
                add_rmsnorm(self.x, self.x, self.xb, self.output_norm, c.dim, c.eps, B, stream=s)
        gemm(t["output"], self.output, self.x, self.logits, B, c.vocab, c.dim, stream=s)
        if greedy:
            argmax(self.logits, c.vocab, B, self.tokens, self.history, self.step_no, stream=s)
            decode_advance(self.pos, self.step_no, stream=s)

    def capture(self) -> None:
        """Capture one greedy step in a CUDA graph (after one eager warm-up step
        that loads the kernels; the caller resets the state afterwards)."""
        import torch
        with torch.cuda.stream(self.stream):
            self.step()
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.step()

    def reset(self, tokens, pos: int = 0) -> None:
        """Set the current tokens and position (ordered on the decode stream)."""
        import torch
        with torch.cuda.stream(self.stream):
            self.tokens.copy_(torch.as_tensor(np.asarray(tokens, np.int32)).to(self.device))
            self.pos.fill_(pos)
            self.step_no.fill_(0)
        self.steps_issued = 0

    def generate(self, n: int) -> None:
        """n greedy steps (graph replays when captured) on self.stream."""
        import torch
        if self.steps_issued + n > self.max_steps:
            raise ValueError(f"more than max_steps={self.max_steps} steps since reset()")
        self.steps_issued += n
        with torch.cuda.stream(self.stream):
            for _ in range(n):
                if self.graph is not None:
                    self.graph.replay()
                else:
                    self.step()

    def fill_kv(self, n_pos: int, seed: int = 1) -> None:
        """Synthetic context: random K/V for positions < n_pos, position = n_pos
        (decode timing after a prefill of n_pos tokens)."""
        import torch
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        with torch.cuda.stream(self.stream):
            self.kcache[:, :, :n_pos].normal_(generator=g)
            self.vcache[:, :, :n_pos].normal_(generator=g)
            self.pos.fill_(n_pos)
