"""Device-resident Llama decode around the quantized GEMVs.

`LlamaDecoder` runs the reference's decode forward (Model::forward,
src/model.h:257-543, dense Llama path) entirely on one GPU through libswq:
embedding row, per layer RMSNorm, q/k/v GEMVs, RoPE + KV-cache append,
grouped-query attention, o GEMV, residual, RMSNorm, gate+up GEMV, SiLU-mul,
down GEMV, residual; final RMSNorm, LM-head GEMV and greedy argmax.  Matrices
of one type that read the same input are stacked into one GEMV (q with k,
gate with up), and every residual add runs in one pass with the RMSNorm
after it (optionally inside the projection that reads the norm).  `rows`
sequences decode in step.  The position lives in device memory, so one
decode step is captured once in a CUDA graph and replayed per token.

Weights are GGUF blocks in device memory: either given (host arrays, for the
tests) or synthetic -- seeded random blocks with the benchmark's value
distributions, generated on the device -- in the Q4_K_M mix (Q6_K for attn_v,
ffn_down and the output matrix, Q4_K elsewhere).

Tensor parallelism (one process per GPU, `group` of G ranks): rank r keeps
query heads [r H/G, (r+1) H/G) and kv heads [r Hkv/G, ...) -- the rows of
wq, wk, wv -- its FFN columns (ffn_split: ffn/G each, or whole 16-byte
row units when ffn/G columns of w_down are not) as rows of gate and up and
columns of w_down, columns [r H hd/G, ...) of wo, and rows [r V/G, ...) of the
LM head.
Attention is local to the rank's heads; the o and down projections give
partial sums that one all-reduce each completes; the rank's slice of the
logits is all-gathered before the argmax.  Every collective is issued on the
decode stream, so the step with its collectives is captured in one graph.
The reference runs one process (no tensor parallelism); a G-rank decoder is
checked against the same model on one rank.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from . import lib as _lib_mod  # noqa: F401  (module import for the ctypes table)
from .lib import (ACT_NONE, ACT_RMSNORM, ACT_SWIGLU, OPT_TENSOR_CORE_MIN_M, add, argmax, add_rmsnorm, gdn_step,
                  attention_decode, attention_prefill, attention_workspace_bytes, decode_advance, dequant, embed,
                  gemm_act_ws, gemm_workspace_bytes, get_option, qkv_bias_norm, rmsnorm, rope_kv, rope_kv_prefill,
                  silu_mul)
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
    # per layer, the types of its seven matrices when they differ between
    # layers (a GGUF Q4_K_M file keeps attn_v / ffn_down in Q6_K on some
    # layers only); None: every layer has `types`
    layer_types: tuple | None = None
    # mixture of experts (0: the dense FFN above): n_experts routed experts of
    # intermediate expert_ffn, top_k per token (softmax over the k router
    # logits), plus a shared expert of shared_ffn (0: none); expert types in
    # types["w_{gate,up,down}_exps"] and types["w_{gate,up,down}_shexp"]
    n_experts: int = 0
    top_k: int = 0
    expert_ffn: int = 0
    shared_ffn: int = 0
    # GatedDeltaNet (linear attention) layers of a hybrid model (Qwen3.5,
    # src/model.h:369-513): their indices, key / value heads and head dims,
    # conv1d width; their matrices (w_qkv, w_z, w_beta, w_alpha, w_dt,
    # w_ssm_out, then the FFN) come from layer_types
    linear_layers: tuple = ()
    lin_n_k: int = 0
    lin_n_v: int = 0
    lin_k_hd: int = 0
    lin_v_hd: int = 0
    lin_conv: int = 0

    @classmethod
    def llama3_70b(cls, **kw) -> "LlamaConfig":
        """Llama-3-70B shape: 80 layers, hidden 8192, 64 query / 8 kv heads of
        128, FFN 28672, vocab 128256."""
        return cls(n_layers=80, dim=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672, vocab=128256, **kw)

    @classmethod
    def moe_40l(cls, **kw) -> "LlamaConfig":
        """The MoE decoder shape: 40 layers, hidden 2048, 16 query / 4 kv heads
        of 128, 256 routed experts of intermediate 512 with top-8 routing and
        one shared expert of 512 (experts in Q4_K), vocab 151936."""
        types = {"wq": Q4_K, "wk": Q4_K, "wv": Q6_K, "wo": Q4_K, "output": Q6_K,
                 "w_gate_exps": Q4_K, "w_up_exps": Q4_K, "w_down_exps": Q4_K,
                 "w_gate_shexp": Q4_K, "w_up_shexp": Q4_K, "w_down_shexp": Q4_K}
        return cls(n_layers=40, dim=2048, n_heads=16, n_kv_heads=4, head_dim=128, ffn=512, vocab=151936,
                   theta=1e6, types=types, n_experts=256, top_k=8, expert_ffn=512, shared_ffn=512, **kw)

    @property
    def is_moe(self) -> bool:
        return self.n_experts > 0

    @property
    def is_hybrid(self) -> bool:
        return len(self.linear_layers) > 0

    @property
    def lin_key_dim(self) -> int:
        return self.lin_n_k * self.lin_k_hd

    @property
    def lin_value_dim(self) -> int:
        return self.lin_n_v * self.lin_v_hd

    def layer_shapes(self, layer: int) -> dict:
        """name -> (N, K) of every quantized matrix layer `layer` may have: a
        GatedDeltaNet layer's projections (w_z, w_beta, w_alpha, w_dt are
        optional) and FFN, else shapes()."""
        if layer not in self.linear_layers:
            return self.shapes()
        kd, vd, nv, H = self.lin_key_dim, self.lin_value_dim, self.lin_n_v, self.dim
        return {"w_qkv": (2 * kd + vd, H), "w_z": (vd, H), "w_beta": (nv, H), "w_alpha": (nv, H),
                "w_dt": (nv, H), "w_ssm_out": (H, vd),
                "w_gate": (self.ffn, H), "w_up": (self.ffn, H), "w_down": (H, self.ffn)}

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def shapes(self) -> dict:
        """name -> (N rows, K columns) of every quantized matrix of a layer
        (for a MoE layer: the attention matrices; the experts are moe_shapes)."""
        att = {"wq": (self.q_dim, self.dim), "wk": (self.kv_dim, self.dim), "wv": (self.kv_dim, self.dim),
               "wo": (self.dim, self.q_dim)}
        if self.is_moe:
            return att
        return dict(att, w_gate=(self.ffn, self.dim), w_up=(self.ffn, self.dim), w_down=(self.dim, self.ffn))

    def moe_shapes(self) -> dict:
        """name -> (N rows, K columns) of one expert's matrices (routed, then shared)."""
        F, Fs, H = self.expert_ffn, self.shared_ffn, self.dim
        return {"w_gate_exps": (F, H), "w_up_exps": (F, H), "w_down_exps": (H, F),
                "w_gate_shexp": (Fs, H), "w_up_shexp": (Fs, H), "w_down_shexp": (H, Fs)}

    def layer_type_map(self, layer: int) -> dict:
        """GGML type of each of layer `layer`'s matrices."""
        if self.layer_types:
            return self.layer_types[layer]
        names = list(self.shapes()) + (list(self.moe_shapes()) if self.is_moe else [])
        return {k: self.types[k] for k in names}

    def weight_bytes_per_token(self) -> int:
        """Quantized weight bytes one decode step reads (all layers + LM head;
        for a MoE model the attention, shared experts and LM head, without the
        routed experts, whose share depends on the routing)."""
        per_layer = [sum(n * row_bytes(self.layer_type_map(li)[k], kk) for k, (n, kk) in
                         self.layer_shapes(li).items() if k in self.layer_type_map(li))
                     for li in range(self.n_layers)]
        if self.is_moe and self.shared_ffn:
            per_layer = [b + sum(n * row_bytes(self.types[k], kk) for k, (n, kk) in self.moe_shapes().items()
                                 if k.endswith("shexp")) for b in per_layer]
        return sum(per_layer) + self.vocab * row_bytes(self.types["output"], self.dim)

    def expert_bytes(self) -> int:
        """Bytes of one routed expert's three matrices."""
        return sum(n * row_bytes(self.types[k], kk) for k, (n, kk) in self.moe_shapes().items()
                   if k.endswith("exps"))


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


# the optional per-layer tensors applied between the q/k/v projections and RoPE
_EXTRAS = frozenset(("bq", "bk", "bv", "q_norm", "k_norm"))


def _upload(host: np.ndarray, device):
    """Host array -> device tensor.  A read-only array (a view of a memory-mapped
    GGUF file) is uploaded from the mapping itself, without a host copy; torch
    only reads it."""
    import warnings

    import torch
    with warnings.catch_warnings():
        warnings.filterwarnings("ignore", message="The given NumPy array is not writable")
        return torch.from_numpy(host).to(device)


def _align_elems(type_id: int) -> int:
    """Fewest whole blocks, in elements, whose bytes are a multiple of 16."""
    qk, bb = LAYOUT[type_id][:2]
    return (16 // math.gcd(bb, 16)) * qk


def ffn_split(cfg: LlamaConfig, world: int) -> list[tuple[int, int]]:
    """FFN columns [f0, f0 + n) of each tensor-parallel rank: the rows of its
    gate/up shard and the columns of its w_down shard.

    Even (ffn / world each) when every rank's w_down rows then start on a
    16-byte boundary, so that the GEMV and GEMM stream them with bulk copies.
    Otherwise (e.g. Q6_K w_down of the 70B shape over 4 or 8 ranks: 28672 / 8
    = 3584 columns = 2940 bytes per row) the FFN is split into whole alignment
    units -- the fewest blocks whose bytes are a multiple of 16, for every
    layer's w_down type -- as evenly as they go, the first ranks taking one
    more (28672 over 8: six ranks of 4096, two of 2048).  Falls back to the even
    split when there are fewer units than ranks."""
    even = [(r * (cfg.ffn // world), cfg.ffn // world) for r in range(world)]
    if world == 1 or cfg.is_moe:
        return even
    unit = 1
    for layer in range(cfg.n_layers):
        a = _align_elems(cfg.layer_type_map(layer)["w_down"])
        unit = unit * a // math.gcd(unit, a)
    if (cfg.ffn // world) % unit == 0 or cfg.ffn % unit:
        return even
    units = cfg.ffn // unit
    base, extra = divmod(units, world)
    if base == 0:
        return even
    out, f0 = [], 0
    for r in range(world):
        n = (base + (1 if r < extra else 0)) * unit
        out.append((f0, n))
        f0 += n
    return out


def _shard(host, type_id: int, N: int, K: int, rows: tuple[int, int] | None, cols: tuple[int, int] | None):
    """Rows [r0, r1) or columns [k0, k1) (whole blocks) of an N x K block matrix."""
    qk, bb = LAYOUT[type_id][:2]
    b = np.asarray(host).reshape(N, (K // qk) * bb)
    if rows is not None:
        b = b[rows[0]:rows[1]]
    if cols is not None:
        b = b[:, (cols[0] // qk) * bb:(cols[1] // qk) * bb]
    return np.ascontiguousarray(b)


class LlamaDecoder:
    def __init__(self, cfg: LlamaConfig, rows: int = 1, device="cuda", seed: int = 0, weights: dict | None = None,
                 max_steps: int = 4096, group=None, weights_from: "LlamaDecoder | None" = None,
                 collective: str = "peer", fuse: tuple | str = "auto", ep_group=None, moe_max_tokens: int = 0):
        """weights: None for synthetic weights, else host arrays: 'token_embd'
        [vocab, dim] fp32 (or (GGML type, blocks)), 'output_norm' [dim], 'output'
        blocks, and per layer 'layers'[l] with 'attn_norm', 'ffn_norm' [dim]
        fp32 and the blocks of wq wk wv wo w_gate w_up w_down (whole matrices;
        each rank keeps its shard), optionally the biases 'bq' [q_dim], 'bk',
        'bv' [kv_dim] and the head norms 'q_norm', 'k_norm' [head_dim].  group: torch.distributed group for tensor parallelism (None:
        this process alone, whatever process groups exist).
        weights_from: a decoder of the same config and group whose device
        weights this one shares (another batch size of the same model).
        collective: "peer" (libswq's one-shot all-reduce over peer memory)
        or "nccl" (torch.distributed.all_reduce) for the o/down sums.
        fuse: activation transforms run inside the projection that reads them
        (swq_gemm_act) instead of as their own pass -- "rmsnorm" (with the
        residual add), "swiglu".  "auto": RMSNorm inside the projections when
        the tensor-core GEMM serves them (one CTA per row converts the
        activations), nothing on the GEMV path (every GEMV CTA would repeat
        the whole row's transform; measured slower), SwiGLU never (slower on
        both paths).

        A MoE config (cfg.n_experts > 0) runs each layer's FFN as swq.moe.MoEFFN:
        routed experts (expert-parallel over ep_group: every rank decodes its
        own rows with the whole attention, and the experts are sharded), plus
        the shared expert.  Host weights of a MoE layer: 'router' [n_experts,
        dim] fp32 and the blocks of w_{gate,up,down}_exps (the experts stacked,
        expert e at rows e*N ..) and w_{gate,up,down}_shexp.  moe_max_tokens:
        rows per MoE call (prefill runs in chunks of it; default max(rows,
        512)); every rank of ep_group must make the same calls (same rows and
        prompt lengths)."""
        import torch
        from .parallel import _world
        self.cfg, self.rows, self.device = cfg, rows, torch.device(device)
        self.group = group
        if cfg.is_moe and group is not None:
            raise ValueError("a MoE decoder runs its attention per rank: shard the experts with ep_group")
        if cfg.is_hybrid and (group is not None or cfg.is_moe or weights is None):
            raise ValueError("a hybrid (GatedDeltaNet) decoder runs on one GPU, dense, from given weights")
        self.ep_group = ep_group
        self.moe_max_tokens = int(moe_max_tokens) or max(rows, 512)
        self.rank, self.world = _world(group) if group is not None else (0, 1)
        G, r = self.world, self.rank
        for what, n in (("query heads", cfg.n_heads), ("kv heads", cfg.n_kv_heads), ("ffn", cfg.ffn),
                        ("vocab", cfg.vocab)):
            if n % G:
                raise ValueError(f"{what}={n} does not split over {G} ranks")
        self.nh, self.nkv = cfg.n_heads // G, cfg.n_kv_heads // G
        self.q_dim, self.kv_dim = self.nh * cfg.head_dim, self.nkv * cfg.head_dim
        self.ffn_off, self.ffn = ffn_split(cfg, G)[r]
        self.vocab = cfg.vocab // G
        dev = self.device
        g = torch.Generator(device=dev)
        g.manual_seed(seed + 1000003 * r)
        f32 = dict(dtype=torch.float32, device=dev)
        # local (rows, K) of every matrix, and the slice of the whole matrix it is
        # this rank's rows (column-parallel) or columns (row-parallel): (first, count)
        row_part = {"wq": (r * self.q_dim, self.q_dim), "wk": (r * self.kv_dim, self.kv_dim),
                    "wv": (r * self.kv_dim, self.kv_dim), "w_gate": (self.ffn_off, self.ffn),
                    "w_up": (self.ffn_off, self.ffn), "output": (r * self.vocab, self.vocab)}
        col_part = {"wo": (r * self.q_dim, self.q_dim), "w_down": (self.ffn_off, self.ffn)}

        def blocks(name, N, K, host, type_id):
            if name in row_part:
                f, n = row_part[name]
                Nl, Kl, rs, cs = n, K, (f, f + n), None
            else:
                f, k = col_part[name]
                Nl, Kl, rs, cs = N, k, None, (f, f + k)
            if host is not None:
                part = _shard(host, type_id, N, K, rs, cs) if G > 1 else np.ascontiguousarray(host)
                return _upload(part.reshape(-1), dev)
            return synthetic_blocks(type_id, Nl, Kl, g, dev)

        W = weights or {}
        if weights_from is not None:
            if weights_from.cfg != cfg or weights_from.world != G:
                raise ValueError("weights_from must have the same config and group size")
            for name in ("token_embd", "output_norm", "output", "fuse_gate_up", "fuse_qk", "layers", "freqs",
                         "moe_base"):
                setattr(self, name, getattr(weights_from, name, None))
            if self.moe_base is not None:
                self.moe_max_tokens = self.moe_base.max_tokens
        else:
            self._load_weights(cfg, W, weights, blocks, g, f32)
        self._alloc_state(cfg, rows, max_steps, f32)
        if collective not in ("peer", "nccl"):
            raise ValueError(f"collective must be 'peer' or 'nccl', not {collective!r}")
        self.collective = collective
        if fuse == "auto":
            fuse = ("rmsnorm",) if rows >= get_option(OPT_TENSOR_CORE_MIN_M) and not (cfg.is_moe or cfg.is_hybrid) \
                else ()
        if (cfg.is_moe or cfg.is_hybrid) and fuse:
            raise ValueError("a MoE or hybrid decoder runs its norms as their own pass (fuse=())")
        if not set(fuse) <= {"rmsnorm", "swiglu"}:
            raise ValueError(f"fuse takes 'rmsnorm' and 'swiglu', not {fuse!r}")
        self.fuse = tuple(fuse)
        self._peer = None
        if G > 1 and collective == "peer":
            from .comm import shared_peer_allreduce
            self._peer = shared_peer_allreduce(rows * cfg.dim, group=group, device=dev)
            self.all_reduce = lambda t: self._peer(t, stream=self.stream)

    @classmethod
    def from_gguf(cls, path, rows: int = 1, context_override: int = 0, **kw) -> "LlamaDecoder":
        """A decoder of the dense Llama-family GGUF file at `path`: its config
        and type mix read as the reference's Model::load does, every projection
        uploaded in its GGUF blocks straight from the memory-mapped file, a
        quantized embedding table dequantized on the device.  The KV cache
        holds the file's context length, capped as the reference caps it
        (context_override when smaller; 4096 when none is given and the file's
        exceeds 8192).  Other keywords as the constructor's."""
        from .gguf import llama_from_gguf
        cfg, W, g = llama_from_gguf(path, context_override)
        try:
            return cls(cfg, rows=rows, weights=W, **kw)
        finally:
            del W
            g.close()

    def _load_weights(self, cfg, W, weights, blocks, g, f32):
        import torch
        dev = self.device
        t = cfg.types
        if weights and isinstance(W["token_embd"], tuple):
            # (GGML type, blocks) of a quantized embedding table: dequantized on
            # the device (bit-exact, as the reference dequantizes it at load,
            # src/model.h:771-772), then ordered before the decode stream's use
            type_id, tb = W["token_embd"]
            self.token_embd = torch.empty((cfg.vocab, cfg.dim), **f32)
            dequant(type_id, _upload(np.ascontiguousarray(tb).reshape(-1), dev), self.token_embd,
                    cfg.vocab * cfg.dim)
            torch.cuda.current_stream(dev).synchronize()
        else:
            self.token_embd = (_upload(np.ascontiguousarray(W["token_embd"], np.float32), dev) if weights
                               else torch.randn((cfg.vocab, cfg.dim), generator=g, **f32))
        self.output_norm = (_upload(np.ascontiguousarray(W["output_norm"], np.float32), dev) if weights
                            else 1.0 + 0.01 * torch.randn(cfg.dim, generator=g, **f32))
        self.output = blocks("output", cfg.vocab, cfg.dim, W.get("output"), t["output"])
        lts = [cfg.layer_type_map(layer) for layer in range(cfg.n_layers)]
        self.fuse_gate_up = all(lt.get("w_gate") == lt.get("w_up") for lt in lts)
        self.fuse_qk = all(lt.get("wq") == lt.get("wk") for lt in lts)
        self.layers = []
        for layer, lt in enumerate(lts):
            lw = W["layers"][layer] if weights else {}
            L = {"types": lt}
            for name in ("attn_norm", "ffn_norm"):
                L[name] = (_upload(np.ascontiguousarray(lw[name], np.float32), dev) if weights
                           else 1.0 + 0.01 * torch.randn(cfg.dim, generator=g, **f32))
            if layer in cfg.linear_layers:
                self._load_linear_layer(cfg, L, lt, lw)
                self.layers.append(L)
                continue
            for name, (N, K) in cfg.shapes().items():
                L[name] = blocks(name, N, K, lw.get(name), lt[name])
            # optional q/k/v biases and q/k head norms (Qwen-style files,
            # src/model.h:291-318): this rank's heads of each bias, the
            # [head_dim] norms whole
            r = self.rank
            for name, n in (("bq", self.q_dim), ("bk", self.kv_dim), ("bv", self.kv_dim)):
                if lw.get(name) is not None:
                    L[name] = _upload(np.ascontiguousarray(np.asarray(lw[name], np.float32)[r * n:(r + 1) * n]), dev)
            for name in ("q_norm", "k_norm"):
                if lw.get(name) is not None:
                    L[name] = _upload(np.ascontiguousarray(lw[name], np.float32), dev)
            if cfg.is_moe:
                L["moe"] = self._moe_layer(cfg, lt, lw if weights else None, layer)
            elif lt["w_gate"] == lt["w_up"]:  # rows of gate then rows of up: one GEMV
                L["w_gate_up"] = torch.cat([L.pop("w_gate"), L.pop("w_up")])
            if lt["wq"] == lt["wk"]:  # rows of q then rows of k
                L["w_qk"] = torch.cat([L.pop("wq"), L.pop("wk")])
            self.layers.append(L)
        self.freqs = torch.from_numpy(rope_freqs(cfg)).to(dev)

    def _load_linear_layer(self, cfg, L, lt, lw) -> None:
        """A GatedDeltaNet layer's projections (whole matrices: the hybrid
        decoder runs on one GPU), its F32 vectors (ssm_a [n_v], conv1d
        [value_dim, conv], ssm_norm [value_dim], each optional as the
        reference's tensors are) and its dense FFN."""
        import torch
        dev = self.device
        for name in ("w_qkv", "w_z", "w_beta", "w_alpha", "w_dt", "w_ssm_out", "w_gate", "w_up", "w_down"):
            if name in lt:
                L[name] = _upload(np.ascontiguousarray(lw[name]).reshape(-1), dev)
        for name in ("ssm_a", "conv1d", "ssm_norm"):
            if lw.get(name) is not None:
                L[name] = _upload(np.ascontiguousarray(lw[name], np.float32).reshape(-1), dev)
        if lt["w_gate"] == lt["w_up"]:
            L["w_gate_up"] = torch.cat([L.pop("w_gate"), L.pop("w_up")])

    def _moe_layer(self, cfg, lt, lw, layer):
        """The MoE FFN of one layer: host weights (lw) or synthetic blocks
        generated on the device (this rank's experts from a rank-dependent
        seed; the router and the shared expert the same on every rank)."""
        import torch
        from .moe import MoEFFN, _group_rank_world
        from .synth import row_bytes
        dev, H, F, E, k = self.device, cfg.dim, cfg.expert_ffn, cfg.n_experts, cfg.top_k
        types = (lt["w_gate_exps"], lt["w_up_exps"], lt["w_down_exps"])
        stypes = (lt["w_gate_shexp"], lt["w_up_shexp"], lt["w_down_shexp"]) if cfg.shared_ffn else None
        base = getattr(self, "moe_base", None)
        kw = dict(group=self.ep_group, device=dev, scratch_from=base, shared_types=stypes, shared_F=cfg.shared_ffn)
        if lw is not None:
            def split(name, n, kk):
                b = np.asarray(lw[name]).reshape(E, n * row_bytes(lt[name], kk))
                return [b[e] for e in range(E)]
            gs, us, ds = (split(nm, *cfg.moe_shapes()[nm]) for nm in ("w_gate_exps", "w_up_exps", "w_down_exps"))
            shared = tuple(np.asarray(lw[nm]) for nm in ("w_gate_shexp", "w_up_shexp", "w_down_shexp")) \
                if cfg.shared_ffn else None
            moe = MoEFFN(list(zip(gs, us, ds)), types, H, F, np.asarray(lw["router"], np.float32), k,
                         self.moe_max_tokens, shared=shared, **kw)
        else:
            ep_rank, ep_world = _group_rank_world(self.ep_group) if self.ep_group is not None else (0, 1)
            el = E // ep_world
            ge = torch.Generator(device=dev)
            ge.manual_seed(7919 * (layer + 1) + 104729 * ep_rank)
            gu_all = synthetic_blocks(types[0], el * 2 * F, H, ge, dev)
            d_all = synthetic_blocks(types[2], el * H, F, ge, dev)
            gr = torch.Generator(device=dev)
            gr.manual_seed(15485863 + layer)
            router = torch.randn(E, H, generator=gr, device=dev) * 0.02
            shared = None
            if cfg.shared_ffn:
                Fs = cfg.shared_ffn
                shared = (synthetic_blocks(stypes[0], Fs, H, gr, dev), synthetic_blocks(stypes[1], Fs, H, gr, dev),
                          synthetic_blocks(stypes[2], H, Fs, gr, dev))
            moe = MoEFFN(None, types, H, F, router, k, self.moe_max_tokens, shared=shared, n_experts=E,
                         device_blocks=(gu_all, d_all), **kw)
        if base is None:
            self.moe_base = moe
        return moe

    def _alloc_state(self, cfg, rows, max_steps, f32):
        import torch
        dev, G = self.device, self.world
        B = rows
        self.x = torch.zeros((B, cfg.dim), **f32)
        self.x2 = torch.zeros_like(self.x)    # fused norms: the residual stream alternates between x and x2
        self.xb = torch.zeros_like(self.x)    # output of the o / down projection (added to the residual)
        self.xn = torch.zeros_like(self.x)    # the normalized input of the next projection
        self.qk = torch.zeros((B, self.q_dim + self.kv_dim), **f32)  # q then k, per row
        self.v = torch.zeros((B, self.kv_dim), **f32)
        self.att = torch.zeros((B, self.q_dim), **f32)
        self.gu = torch.zeros((B, 2 * self.ffn), **f32)
        self.h = torch.zeros((B, self.ffn), **f32)
        self.logits = torch.zeros((B, cfg.vocab), **f32)
        if G > 1:
            self.logits_l = torch.zeros((B, self.vocab), **f32)       # this rank's slice
            self.logits_g = torch.zeros((G, B, self.vocab), **f32)    # all slices, rank-major
        self.kcache = torch.zeros((cfg.n_layers, B, cfg.max_seq, self.kv_dim), **f32)
        self.vcache = torch.zeros_like(self.kcache)
        self.tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.step_no = torch.zeros(1, dtype=torch.int32, device=dev)
        self.history = torch.zeros((max_steps, B), dtype=torch.int32, device=dev)
        if cfg.is_hybrid:
            kd, vd, nv = cfg.lin_key_dim, cfg.lin_value_dim, cfg.lin_n_v
            self.gdn_qkv = torch.zeros((B, 2 * kd + vd), **f32)
            self.gdn_z = torch.zeros((B, vd), **f32)
            self.gdn_gates = torch.zeros((3, B, nv), **f32)  # beta, alpha, dt projections
            self.gdn_y = torch.zeros((B, vd), **f32)
            nlin = len(cfg.linear_layers)
            self.gdn_state = torch.zeros((nlin, B, nv, cfg.lin_k_hd, cfg.lin_v_hd), **f32)
            self.gdn_conv = torch.zeros((nlin, B, vd, max(1, cfg.lin_conv)), **f32)
        self.ws_bytes = attention_workspace_bytes(self.nh, self.nkv, cfg.head_dim, B, cfg.max_seq)
        self.ws = torch.zeros(max(1, self.ws_bytes // 4), **f32)  # zero-filled, as the kernel expects
        self.gemm_ws, self.gemm_ws_bytes = None, 0  # tensor-core GEMM scratch, grown on first need
        self.max_steps = max_steps
        self.steps_issued = 0
        self.stream = torch.cuda.Stream(device=dev)
        self.graph = None
        self.all_reduce = self._nccl_all_reduce

    # ------------------------------------------------------------ collectives
    def _nccl_all_reduce(self, t) -> None:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _gather_logits(self) -> None:
        import torch.distributed as dist
        dist.all_gather_into_tensor(self.logits_g, self.logits_l, group=self.group)
        self.logits.view(self.rows, self.world, self.vocab).copy_(self.logits_g.transpose(0, 1))

    # ------------------------------------------------------------ one token
    def _gemm(self, type_id, W, X, Y, M, N, K, stream, kind=ACT_NONE, residual=None, norm_w=None, sum_out=None,
              ld=0):
        # The tensor-core GEMM's scratch is this decoder's own workspace: a
        # captured step allocates nothing, and two decoders on one device never
        # share scratch.  Every call of this decoder runs on its one stream.
        need = gemm_workspace_bytes(type_id, M, N, K)
        if need > self.gemm_ws_bytes:
            import torch
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(f"GEMM workspace of {self.gemm_ws_bytes} bytes, a captured call needs {need}")
            self.stream.synchronize()  # the old workspace may still be read by queued kernels
            self.gemm_ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            self.gemm_ws_bytes = need
        gemm_act_ws(type_id, W, X, Y, M, N, K, self.gemm_ws, self.gemm_ws_bytes, kind=kind, residual=residual,
                    norm_w=norm_w, eps=self.cfg.eps, sum_out=sum_out, ld=ld, stream=stream)

    def step(self, greedy: bool = True) -> None:
        """One decode step for all rows at position *pos: logits of the current
        tokens; with greedy, tokens <- argmax (also into history) and pos += 1.

        The residual stream is x; d holds the output of the last o or down
        projection, added to x by the RMSNorm pass that follows it (or, with
        fuse=("rmsnorm",), by the projection that reads the norm, which then
        writes the sum to x2 and the stream alternates between x and x2)."""
        c, B, s = self.cfg, self.rows, self.stream
        gemm = self._gemm  # noqa: F811
        qd, kvd, ffn = self.q_dim, self.kv_dim, self.ffn
        tp = self.world > 1
        ld = qd + kvd
        q, k = self.qk, self.qk[:, qd:]
        fuse_rms, fuse_glu = "rmsnorm" in self.fuse, "swiglu" in self.fuse
        x, x2, d, xb = self.x, self.x2, self.xb, self.xn
        embed(x, self.token_embd, self.tokens, c.dim, c.vocab, B, stream=s)
        if not fuse_rms:
            rmsnorm(xb, x, self.layers[0]["attn_norm"], c.dim, c.eps, B, stream=s)
        pending = None  # fused: d to add to the residual before the next norm
        for li, L in enumerate(self.layers):
            t = L["types"]
            if li in c.linear_layers:  # GatedDeltaNet: norm(x) -> d (fuse=() for hybrid models)
                self._gdn_layer(li, L, xb, d)
            else:
                # q, k, v of norm(x) (fused: x2 = x + pending first)
                if fuse_rms:
                    src, a_in = x, dict(kind=ACT_RMSNORM, residual=pending, norm_w=L["attn_norm"])
                    a_qk = dict(a_in, sum_out=x2)
                else:
                    src, a_in, a_qk = xb, {}, {}
                if "w_qk" in L:
                    gemm(t["wq"], L["w_qk"], src, self.qk, B, ld, c.dim, stream=s, **a_qk)
                else:
                    gemm(t["wq"], L["wq"], src, self.att, B, qd, c.dim, stream=s, **a_qk)
                    q[:, :qd].copy_(self.att)
                    gemm(t["wk"], L["wk"], src, self.v, B, kvd, c.dim, stream=s, **a_in)
                    k.copy_(self.v)
                gemm(t["wv"], L["wv"], src, self.v, B, kvd, c.dim, stream=s, **a_in)
                if _EXTRAS.intersection(L):
                    qkv_bias_norm(q, k, self.v, L.get("bq"), L.get("bk"), L.get("bv"), L.get("q_norm"),
                                  L.get("k_norm"), qd, kvd, c.head_dim, c.eps, B, ldq=ld, ldk=ld, ldv=kvd, stream=s)
                kc, vc = self.kcache[li], self.vcache[li]
                rope_kv(q, k, self.v, kc, vc, self.pos, self.freqs, qd, kvd, c.head_dim, c.head_dim,
                        c.rope_neox, B, c.max_seq, ldq=ld, ldk=ld, stream=s)
                attention_decode(self.att, q, kc, vc, self.pos, self.ws, self.ws_bytes, self.nh, self.nkv,
                                 c.head_dim, B, c.max_seq, ldq=ld, stream=s)
                gemm(t["wo"], L["wo"], self.att, d, B, c.dim, qd, stream=s)
            if tp:
                self.all_reduce(d)
            # gate, up of norm(residual + o)
            if fuse_rms:
                src, a_in = x2, dict(kind=ACT_RMSNORM, residual=d, norm_w=L["ffn_norm"])
                a_g = dict(a_in, sum_out=x)
            else:
                add_rmsnorm(xb, x, d, L["ffn_norm"], c.dim, c.eps, B, stream=s)  # x += o; xb = norm(x)
                src, a_in, a_g = xb, {}, {}
            if "moe" in L:  # routed experts + shared expert of norm(x) into d
                L["moe"](xb, B, out=d, peer_tokens=B, stream=s)
            elif "w_gate_up" in L:
                gemm(t["w_gate"], L["w_gate_up"], src, self.gu, B, 2 * ffn, c.dim, stream=s, **a_g)
            else:
                gemm(t["w_gate"], L["w_gate"], src, self.h, B, ffn, c.dim, stream=s, **a_g)
                self.gu[:, :ffn].copy_(self.h)
                gemm(t["w_up"], L["w_up"], src, self.h, B, ffn, c.dim, stream=s, **a_in)
                self.gu[:, ffn:].copy_(self.h)
            if "moe" in L:
                pass
            elif fuse_glu:
                gemm(t["w_down"], L["w_down"], self.gu, d, B, c.dim, ffn, stream=s, kind=ACT_SWIGLU, ld=2 * ffn)
            else:
                silu_mul(self.h, self.gu, self.gu[:, ffn:], ffn, B, 2 * ffn, stream=s)
                gemm(t["w_down"], L["w_down"], self.h, d, B, c.dim, ffn, stream=s)
            if tp:
                self.all_reduce(d)
            if fuse_rms:
                pending = d
            elif li + 1 < len(self.layers):  # x += down; xb = next layer's attention norm of x
                add_rmsnorm(xb, x, d, self.layers[li + 1]["attn_norm"], c.dim, c.eps, B, stream=s)
            else:  # x += down; xb = output norm of x
                add_rmsnorm(xb, x, d, self.output_norm, c.dim, c.eps, B, stream=s)
        if fuse_rms:
            src, a_out = x, dict(kind=ACT_RMSNORM, residual=pending, norm_w=self.output_norm)
        else:
            src, a_out = xb, {}
        t_out = c.types["output"]
        if tp:
            gemm(t_out, self.output, src, self.logits_l, B, self.vocab, c.dim, stream=s, **a_out)
            self._gather_logits()
        else:
            gemm(t_out, self.output, src, self.logits, B, c.vocab, c.dim, stream=s, **a_out)
        if greedy:
            argmax(self.logits, c.vocab, B, self.tokens, self.history, self.step_no, stream=s)
            decode_advance(self.pos, self.step_no, stream=s)

    def _gdn_layer(self, li: int, L: dict, xb, d) -> None:
        """A GatedDeltaNet layer of the step (src/model.h:369-513): the q/k/v,
        gate, beta, alpha and dt projections of norm(x) = xb, swq_gdn_step
        (conv1d, gated delta rule, head norm, gate), the ssm_out projection
        into d."""
        c, B, s, t = self.cfg, self.rows, self.stream, L["types"]
        kd, vd, nv = c.lin_key_dim, c.lin_value_dim, c.lin_n_v
        gemm = self._gemm
        gemm(t["w_qkv"], L["w_qkv"], xb, self.gdn_qkv, B, 2 * kd + vd, c.dim, stream=s)
        if "w_z" in L:
            gemm(t["w_z"], L["w_z"], xb, self.gdn_z, B, vd, c.dim, stream=s)
        gates = []
        for i, name in enumerate(("w_beta", "w_alpha", "w_dt")):
            if name in L:
                gemm(t[name], L[name], xb, self.gdn_gates[i], B, nv, c.dim, stream=s)
            gates.append(self.gdn_gates[i] if name in L else None)
        j = c.linear_layers.index(li)
        gdn_step(self.gdn_qkv, self.gdn_z if "w_z" in L else None, gates[0], gates[1], gates[2], L.get("ssm_a"),
                 L.get("conv1d"), L.get("ssm_norm"), self.gdn_state[j], self.gdn_conv[j], self.gdn_y, B,
                 c.lin_n_k, nv, c.lin_k_hd, c.lin_v_hd, c.lin_conv if "conv1d" in L else 0, stream=s)
        gemm(t["w_ssm_out"], L["w_ssm_out"], self.gdn_y, d, B, c.dim, vd, stream=s)

    def _gdn_prefill(self, li: int, L: dict, xn, d, P: int) -> None:
        """A GatedDeltaNet layer of a prefill: its projections as M = rows x P
        row GEMMs, then the recurrence one prompt position at a time (swq_gdn_step
        on the rows' position p: the reference's Model::forward per token,
        src/model.h:369-513), the ssm_out projection of all positions into d."""
        import torch
        c, B, s, t = self.cfg, self.rows, self.stream, L["types"]
        kd, vd, nv = c.lin_key_dim, c.lin_value_dim, c.lin_n_v
        M, gemm, dev = B * P, self._gemm, self.device
        f32 = dict(dtype=torch.float32, device=dev)
        qkv = torch.empty((M, 2 * kd + vd), **f32)
        gemm(t["w_qkv"], L["w_qkv"], xn, qkv, M, 2 * kd + vd, c.dim, s)
        z = None
        if "w_z" in L:
            z = torch.empty((M, vd), **f32)
            gemm(t["w_z"], L["w_z"], xn, z, M, vd, c.dim, s)
        gates = []
        for name in ("w_beta", "w_alpha", "w_dt"):
            g = None
            if name in L:
                g = torch.empty((M, nv), **f32)
                gemm(t[name], L[name], xn, g, M, nv, c.dim, s)
            gates.append(g)
        y = torch.empty((M, vd), **f32)
        j = c.linear_layers.index(li)
        at_p = lambda a, p: None if a is None else a.view(B, P, -1)[:, p].contiguous()  # noqa: E731
        for p in range(P):
            gdn_step(at_p(qkv, p), at_p(z, p), at_p(gates[0], p), at_p(gates[1], p), at_p(gates[2], p),
                     L.get("ssm_a"), L.get("conv1d"), L.get("ssm_norm"), self.gdn_state[j], self.gdn_conv[j],
                     self.gdn_y, B, c.lin_n_k, nv, c.lin_k_hd, c.lin_v_hd, c.lin_conv if "conv1d" in L else 0,
                     stream=s)
            y.view(B, P, vd)[:, p].copy_(self.gdn_y)
        gemm(t["w_ssm_out"], L["w_ssm_out"], y, d, M, c.dim, vd, s)

    def prefill(self, prompts, pos0: int = 0, all_logits: bool = False):
        """Batched prefill: the prompt tokens of every sequence through the whole
        model at once -- M = rows x P activation rows, every projection one
        M-row tensor-core GEMM, causal attention over each sequence's cache
        (swq_rope_kv_prefill, swq_attention_prefill).  The reference runs a
        prompt as P calls of Model::forward (src/main.cpp:284-287); the logits
        of each position are the same computation.

        prompts: rows lists (or a [rows, P] array) of P token ids, written at
        positions pos0 .. pos0 + P - 1 of each sequence's KV cache.  Afterwards
        the decoder continues from there: self.logits holds the last prompt
        position's logits, tokens = their argmax (also history[0]), pos =
        pos0 + P, and generate() decodes on.  all_logits: also return the
        logits of every prompt position, [rows, P, vocab] (one process)."""
        import torch
        c, B, s = self.cfg, self.rows, self.stream
        toks = np.asarray(prompts, dtype=np.int32)
        if toks.ndim != 2 or toks.shape[0] != B or toks.shape[1] < 1:
            raise ValueError(f"prompts must be {B} lists of at least one token, got shape {toks.shape}")
        P = int(toks.shape[1])
        if pos0 < 0 or pos0 + P > c.max_seq:
            raise ValueError(f"positions {pos0}..{pos0 + P - 1} do not fit max_seq={c.max_seq}")
        if np.any((toks < 0) | (toks >= c.vocab)):
            raise ValueError("token id outside the vocabulary")
        tp = self.world > 1
        if tp and all_logits:
            raise ValueError("all_logits needs the whole vocabulary on one process")
        M, dev, gemm = B * P, self.device, self._gemm
        qd, kvd, ffn, hd = self.q_dim, self.kv_dim, self.ffn, c.head_dim
        ld = qd + kvd
        f32 = dict(dtype=torch.float32, device=dev)
        with torch.cuda.stream(s):
            tok_d = torch.from_numpy(toks.reshape(-1)).to(dev, non_blocking=False)
            x = torch.empty((M, c.dim), **f32)
            xn, d = torch.empty_like(x), torch.empty_like(x)
            qk = torch.empty((M, ld), **f32)
            v = torch.empty((M, kvd), **f32)
            att = torch.empty((M, qd), **f32)
            gu = torch.empty((M, 2 * ffn), **f32)
            h = torch.empty((M, ffn), **f32)
            for r0 in range(0, M, 65535):  # the embedding kernel's grid holds 65535 rows
                r1 = min(M, r0 + 65535)
                embed(x[r0:r1], self.token_embd, tok_d[r0:r1], c.dim, c.vocab, r1 - r0, stream=s)
            rmsnorm(xn, x, self.layers[0]["attn_norm"], c.dim, c.eps, M, stream=s)
            if c.is_hybrid and pos0 == 0:  # new sequences: the recurrences start from zero
                self.gdn_state.zero_()
                self.gdn_conv.zero_()
            for li, L in enumerate(self.layers):
                t = L["types"]
                if li in c.linear_layers:  # GatedDeltaNet: norm(x) -> d
                    self._gdn_prefill(li, L, xn, d, P)
                else:
                    if "w_qk" in L:
                        gemm(t["wq"], L["w_qk"], xn, qk, M, ld, c.dim, s)
                    else:
                        gemm(t["wq"], L["wq"], xn, att, M, qd, c.dim, s)
                        qk[:, :qd].copy_(att)
                        gemm(t["wk"], L["wk"], xn, v, M, kvd, c.dim, s)
                        qk[:, qd:].copy_(v)
                    gemm(t["wv"], L["wv"], xn, v, M, kvd, c.dim, s)
                    if _EXTRAS.intersection(L):
                        qkv_bias_norm(qk, qk[:, qd:], v, L.get("bq"), L.get("bk"), L.get("bv"), L.get("q_norm"),
                                      L.get("k_norm"), qd, kvd, hd, c.eps, M, ldq=ld, ldk=ld, ldv=kvd, stream=s)
                    kc, vc = self.kcache[li], self.vcache[li]
                    rope_kv_prefill(qk, qk[:, qd:], v, kc, vc, pos0, P, self.freqs, qd, kvd, hd, hd, c.rope_neox,
                                    B, c.max_seq, ldq=ld, ldk=ld, ldv=kvd, stream=s)
                    attention_prefill(att, qk, kc, vc, pos0, P, self.nh, self.nkv, hd, B, c.max_seq, ldq=ld,
                                      ldo=qd, stream=s)
                    gemm(t["wo"], L["wo"], att, d, M, c.dim, qd, s)
                    if tp:
                        self._nccl_all_reduce(d)
                add_rmsnorm(xn, x, d, L["ffn_norm"], c.dim, c.eps, M, stream=s)  # x += o; xn = norm(x)
                if "moe" in L:  # in chunks of moe_max_tokens rows, the same on every rank
                    ch = self.moe_max_tokens
                    for r0 in range(0, M, ch):
                        r1 = min(M, r0 + ch)
                        L["moe"](xn[r0:r1], r1 - r0, out=d[r0:r1], peer_tokens=r1 - r0, stream=s)
                else:
                    if "w_gate_up" in L:
                        gemm(t["w_gate"], L["w_gate_up"], xn, gu, M, 2 * ffn, c.dim, s)
                    else:
                        gemm(t["w_gate"], L["w_gate"], xn, h, M, ffn, c.dim, s)
                        gu[:, :ffn].copy_(h)
                        gemm(t["w_up"], L["w_up"], xn, h, M, ffn, c.dim, s)
                        gu[:, ffn:].copy_(h)
                    silu_mul(h, gu, gu[:, ffn:], ffn, M, 2 * ffn, stream=s)
                    gemm(t["w_down"], L["w_down"], h, d, M, c.dim, ffn, s)
                if tp:
                    self._nccl_all_reduce(d)
                if li + 1 < len(self.layers):
                    add_rmsnorm(xn, x, d, self.layers[li + 1]["attn_norm"], c.dim, c.eps, M, stream=s)
                else:
                    add(x, d, M * c.dim, stream=s)
            t_out = c.types["output"]
            every = None
            if all_logits:
                rmsnorm(xn, x, self.output_norm, c.dim, c.eps, M, stream=s)
                every = torch.empty((M, c.vocab), **f32)
                gemm(t_out, self.output, xn, every, M, c.vocab, c.dim, s)
                self.logits.copy_(every.view(B, P, c.vocab)[:, P - 1])
            else:
                x_last = x.view(B, P, c.dim)[:, P - 1].contiguous()
                xl = torch.empty_like(x_last)
                rmsnorm(xl, x_last, self.output_norm, c.dim, c.eps, B, stream=s)
                if tp:
                    gemm(t_out, self.output, xl, self.logits_l, B, self.vocab, c.dim, s)
                    self._gather_logits()
                else:
                    gemm(t_out, self.output, xl, self.logits, B, c.vocab, c.dim, s)
            self.step_no.fill_(0)
            argmax(self.logits, c.vocab, B, self.tokens, self.history, self.step_no, stream=s)
            self.pos.fill_(pos0 + P)
            self.step_no.fill_(1)
        self.steps_issued = 1
        return None if every is None else every.view(B, P, c.vocab)

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
        """Set the current tokens and position (ordered on the decode stream).
        Position 0 starts new sequences: the GatedDeltaNet layers' recurrent
        state and conv history are zeroed, as Model::reset does."""
        import torch
        with torch.cuda.stream(self.stream):
            self.tokens.copy_(torch.as_tensor(np.asarray(tokens, np.int32)).to(self.device))
            self.pos.fill_(pos)
            self.step_no.fill_(0)
            if pos == 0 and self.cfg.is_hybrid:
                self.gdn_state.zero_()
                self.gdn_conv.zero_()
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
