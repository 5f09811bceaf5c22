"""LlamaDecoder's host logic on the CPU: which libswq operations a decode
step, a prefill and a GGUF load issue, with what sizes, strides and buffers.

The device operations are replaced by recorders (no kernel runs) and the
decoder's tensors live on the CPU, so this checks only the wiring: per-layer
GGML types reach the right projections, stacked q/k and gate/up matrices are
used exactly when a layer's types allow it, prefill rows and cache slices are
laid out as the kernels expect, and the decoder's state after a prefill.
The numerics are the GPU tests' (test_gpu_model.py, test_gpu_x_prefill.py,
test_gpu_whole_model_files.py)."""
import contextlib

import numpy as np
import pytest
import torch

import llama_gguf as LG
import swq.model as M
from swq import synth
from test_gpu_model import _small, _weights

OPS = ("embed", "rmsnorm", "add_rmsnorm", "gemm_act_ws", "rope_kv", "attention_decode", "silu_mul", "argmax",
       "qkv_bias_norm", "decode_advance", "rope_kv_prefill", "attention_prefill", "add", "dequant", "gdn_step")


class _Stream:
    def synchronize(self):
        pass


@pytest.fixture
def calls(monkeypatch):
    log = []

    def recorder(name):
        def f(*a, **kw):
            log.append((name, a, kw))
        return f

    for name in OPS:
        monkeypatch.setattr(M, name, recorder(name))
    monkeypatch.setattr(M, "gemm_workspace_bytes", lambda *a: 0)
    monkeypatch.setattr(torch.cuda, "Stream", lambda device=None: _Stream())
    monkeypatch.setattr(torch.cuda, "stream", lambda s: contextlib.nullcontext())
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: _Stream())
    return log


def _gemms(log):
    """(type, weight tensor, M, N, K) of every projection, in order."""
    return [(a[0], a[1], a[4], a[5], a[6]) for name, a, _ in log if name == "gemm_act_ws"]


def _mixed_cfg():
    cfg = _small()
    cfg.layer_types = ({"wq": synth.Q4_K, "wk": synth.Q4_K, "wv": synth.Q6_K, "wo": synth.Q4_K,
                        "w_gate": synth.Q4_K, "w_up": synth.Q4_K, "w_down": synth.Q6_K},
                       {"wq": synth.Q5_K, "wk": synth.Q8_0, "wv": synth.Q8_0, "wo": synth.Q2_K,
                        "w_gate": synth.Q3_K, "w_up": synth.Q4_0, "w_down": synth.Q4_K})
    return cfg


def _weights_for(cfg, seed):
    rng = np.random.default_rng(seed)
    layers = []
    for li in range(cfg.n_layers):
        lt = cfg.layer_type_map(li)
        L = {"attn_norm": np.ones(cfg.dim, np.float32), "ffn_norm": np.ones(cfg.dim, np.float32)}
        for k, (n, kk) in cfg.shapes().items():
            L[k] = synth.random_blocks(lt[k], n, kk, seed=seed + 10 * li + len(L))
        layers.append(L)
    return {"token_embd": rng.standard_normal((cfg.vocab, cfg.dim)).astype(np.float32),
            "output_norm": np.ones(cfg.dim, np.float32),
            "output": synth.random_blocks(cfg.types["output"], cfg.vocab, cfg.dim, seed=seed + 99), "layers": layers}


def test_step_uses_each_layers_types(calls):
    cfg = _mixed_cfg()
    dec = M.LlamaDecoder(cfg, rows=1, device="cpu", weights=_weights_for(cfg, 5))
    assert "w_qk" in dec.layers[0] and "w_gate_up" in dec.layers[0]
    assert "w_qk" not in dec.layers[1] and "w_gate_up" not in dec.layers[1]  # types differ: separate matrices
    dec.step()
    g = _gemms(calls)
    qd, kvd, ffn, dim = dec.q_dim, dec.kv_dim, dec.ffn, cfg.dim
    L0, L1 = dec.layers
    want = [(synth.Q4_K, L0["w_qk"], 1, qd + kvd, dim), (synth.Q6_K, L0["wv"], 1, kvd, dim),
            (synth.Q4_K, L0["wo"], 1, dim, qd), (synth.Q4_K, L0["w_gate_up"], 1, 2 * ffn, dim),
            (synth.Q6_K, L0["w_down"], 1, dim, ffn),
            (synth.Q5_K, L1["wq"], 1, qd, dim), (synth.Q8_0, L1["wk"], 1, kvd, dim),
            (synth.Q8_0, L1["wv"], 1, kvd, dim), (synth.Q2_K, L1["wo"], 1, dim, qd),
            (synth.Q3_K, L1["w_gate"], 1, ffn, dim), (synth.Q4_0, L1["w_up"], 1, ffn, dim),
            (synth.Q4_K, L1["w_down"], 1, dim, ffn), (cfg.types["output"], dec.output, 1, cfg.vocab, dim)]
    assert len(g) == len(want)
    for got, exp in zip(g, want):
        assert got[0] == exp[0] and got[1] is exp[1] and got[2:] == exp[2:], (got[0], got[2:], exp[0], exp[2:])
    # weight bytes per token follow the per-layer mix
    per_layer = [sum(n * synth.row_bytes(cfg.layer_type_map(li)[k], kk) for k, (n, kk) in cfg.shapes().items())
                 for li in range(2)]
    assert cfg.weight_bytes_per_token() == sum(per_layer) + cfg.vocab * synth.row_bytes(cfg.types["output"], dim)


@pytest.mark.parametrize("rows,P,pos0,every", [(1, 7, 0, True), (3, 5, 2, False)])
def test_prefill_wiring(calls, rows, P, pos0, every):
    cfg = _small()
    dec = M.LlamaDecoder(cfg, rows=rows, device="cpu", weights=_weights(cfg, seed=9))
    prompts = [[(5 * r + 3 * p) % cfg.vocab for p in range(P)] for r in range(rows)]
    out = dec.prefill(prompts, pos0=pos0, all_logits=every)
    Mr, qd, kvd, ffn = rows * P, dec.q_dim, dec.kv_dim, dec.ffn
    names = [c[0] for c in calls]
    assert names[0] == "embed" and calls[0][1][5] == Mr
    ropes = [c for c in calls if c[0] == "rope_kv_prefill"]
    atts = [c for c in calls if c[0] == "attention_prefill"]
    assert len(ropes) == len(atts) == cfg.n_layers
    for li, (r, a) in enumerate(zip(ropes, atts)):
        ra, rk = r[1], r[2]
        assert ra[3] is not None and ra[3].data_ptr() == dec.kcache[li].data_ptr()  # this layer's cache
        assert (ra[5], ra[6], ra[8], ra[9], ra[13], ra[14]) == (pos0, P, qd, kvd, rows, cfg.max_seq)
        assert ra[1].data_ptr() == ra[0].data_ptr() + 4 * qd  # k: the columns after q in the same rows
        assert rk == {"ldq": qd + kvd, "ldk": qd + kvd, "ldv": kvd, "stream": dec.stream}
        aa, ak = a[1], a[2]
        assert (aa[4], aa[5], aa[6], aa[7], aa[9], aa[10]) == (pos0, P, dec.nh, dec.nkv, rows, cfg.max_seq)
        assert ak["ldq"] == qd + kvd and ak["ldo"] == qd
    g = _gemms(calls)
    assert all(x[2] == Mr for x in g[:-1])                 # every layer projection has M = rows x P
    assert g[-1][2] == (Mr if every else rows) and g[-1][3] == cfg.vocab
    assert names[-1] == "argmax"
    assert int(dec.pos.item()) == pos0 + P and int(dec.step_no.item()) == 1 and dec.steps_issued == 1
    assert (out is not None) == every and (out is None or tuple(out.shape) == (rows, P, cfg.vocab))


def test_prefill_rejects_bad_prompts(calls):
    cfg = _small()
    dec = M.LlamaDecoder(cfg, rows=2, device="cpu", weights=_weights(cfg, seed=9))
    with pytest.raises(ValueError):
        dec.prefill([[1, 2, 3]])                           # one prompt for two rows
    with pytest.raises(ValueError):
        dec.prefill([[1] * 60, [2] * 60], pos0=10)         # past max_seq = 64
    with pytest.raises(ValueError):
        dec.prefill([[1, cfg.vocab], [2, 3]])              # token id outside the vocabulary
    assert calls == []


def test_from_gguf_wiring(calls, tmp_path):
    """The tied file: a Q8_0 embedding table dequantized on the device (once,
    vocab x dim elements) and used as the LM head; the mix file: every
    layer's projections with its own types."""
    dec = M.LlamaDecoder.from_gguf(LG.write(tmp_path / "t.gguf", "tied"), device="cpu")
    dq = [c for c in calls if c[0] == "dequant"]
    assert len(dq) == 1 and dq[0][1][0] == synth.Q8_0 and dq[0][1][3] == dec.cfg.vocab * dec.cfg.dim
    assert dec.cfg.types["output"] == synth.Q8_0 and dec.output.numel() == dec.cfg.vocab * dec.cfg.dim // 32 * 34
    calls.clear()
    dec = M.LlamaDecoder.from_gguf(LG.write(tmp_path / "m.gguf", "mix"), device="cpu")
    dec.step()
    types = [x[0] for x in _gemms(calls)]
    v = LG.VARIANTS["mix"]["layers"]
    assert types == [v[0]["wq"], v[0]["wv"], v[0]["wo"], v[0]["w_gate"], v[0]["w_down"],
                     v[1]["wq"], v[1]["wv"], v[1]["wo"], v[1]["w_gate"], v[1]["w_down"], synth.Q6_K]


def test_hybrid_prefill_wiring(calls, tmp_path):
    """A hybrid file's prefill: the GatedDeltaNet layer's projections once over
    all rows x P positions, its recurrence (swq_gdn_step) once per position on
    that position's rows, in order, from a zeroed state; the attention layer
    through the prefill kernels."""
    dec = M.LlamaDecoder.from_gguf(LG.write(tmp_path / "h.gguf", "hybrid"), device="cpu", rows=2)
    c = dec.cfg
    dec.gdn_state.fill_(1.0)
    dec.gdn_conv.fill_(1.0)
    calls.clear()
    P = 4
    dec.prefill([[1, 2, 3, 4], [5, 6, 7, 8]])
    assert float(dec.gdn_state.abs().sum()) == 0.0 and float(dec.gdn_conv.abs().sum()) == 0.0
    steps = [a for name, a, _ in calls if name == "gdn_step"]
    assert len(steps) == P * len(c.linear_layers)
    for a in steps:
        assert a[0].shape == (2, 2 * c.lin_key_dim + c.lin_value_dim) and a[11] == 2  # one position, both rows
    g = _gemms(calls)
    assert (g[0][2], g[0][3]) == (2 * P, 2 * c.lin_key_dim + c.lin_value_dim)  # w_qkv over all positions
    assert sum(1 for name, _, _ in calls if name == "attention_prefill") == c.n_layers - len(c.linear_layers)
    assert int(dec.pos.item()) == P


@pytest.mark.parametrize("rank", [0, 1])
def test_tensor_parallel_shards_with_mixed_types(calls, monkeypatch, rank):
    """Rank r of 2 keeps rows [r N/2, (r+1) N/2) of the column-parallel
    matrices and whole blocks of columns [r K/2, (r+1) K/2) of wo and w_down,
    whatever each layer's block size (32 or 256 elements)."""
    import swq.parallel as P
    monkeypatch.setattr(P, "_world", lambda group: (rank, 2))
    cfg = _mixed_cfg()
    W = _weights_for(cfg, 5)
    dec = M.LlamaDecoder(cfg, rows=1, device="cpu", weights=W, group=object(), collective="nccl")
    assert (dec.nh, dec.nkv, dec.ffn, dec.vocab) == (4, 1, 512, 500)
    for li, L in enumerate(dec.layers):
        lt = cfg.layer_type_map(li)
        for key, (N, K) in cfg.shapes().items():
            qk, bb = synth.block_geometry(lt[key])
            full = W["layers"][li][key].reshape(N, K // qk, bb)
            if key in ("wo", "w_down"):
                nb = K // qk // 2
                want = full[:, rank * nb:(rank + 1) * nb]
            else:
                want = full[rank * N // 2:(rank + 1) * N // 2]
            if key in ("wq", "wk") and "w_qk" in L:
                nq = dec.q_dim * synth.row_bytes(lt["wq"], K)
                got = L["w_qk"][:nq] if key == "wq" else L["w_qk"][nq:]
            elif key in ("w_gate", "w_up") and "w_gate_up" in L:
                ng = dec.ffn * synth.row_bytes(lt["w_gate"], K)
                got = L["w_gate_up"][:ng] if key == "w_gate" else L["w_gate_up"][ng:]
            else:
                got = L[key]
            assert np.array_equal(got.numpy(), want.reshape(-1)), (li, key)
    out = W["output"].reshape(cfg.vocab, -1)[rank * 500:(rank + 1) * 500]
    assert np.array_equal(dec.output.numpy(), out.reshape(-1))


def test_tensor_parallel_prefill_collectives(calls, monkeypatch):
    """Two sums per layer (after o and down, on the M-row partial outputs) and
    one gather of the vocab-sharded logits, in that order on every rank."""
    import swq.parallel as P
    monkeypatch.setattr(P, "_world", lambda group: (1, 2))
    cfg = _small()
    dec = M.LlamaDecoder(cfg, rows=2, device="cpu", weights=_weights(cfg, seed=9), group=object(),
                         collective="nccl")
    seen = []
    monkeypatch.setattr(dec, "_nccl_all_reduce", lambda t: seen.append(("sum", tuple(t.shape))))
    monkeypatch.setattr(dec, "_gather_logits", lambda: seen.append(("gather",)))
    dec.prefill([[1, 2, 3], [4, 5, 6]])
    assert seen == [("sum", (6, cfg.dim))] * (2 * cfg.n_layers) + [("gather",)]
    g = _gemms(calls)
    assert g[-1][1] is dec.output and g[-1][2:] == (2, cfg.vocab // 2, cfg.dim)  # this rank's vocab rows
    with pytest.raises(ValueError):
        dec.prefill([[1, 2], [3, 4]], all_logits=True)  # the whole vocabulary lives on no single rank


def test_tensor_parallel_step_collectives(calls, monkeypatch):
    """A decode step on the peer all-reduce: two sums per layer of the
    [rows, dim] partial outputs on the decode stream, then the logits gather."""
    import swq.comm as C
    import swq.parallel as P
    monkeypatch.setattr(P, "_world", lambda group: (0, 2))
    seen = []

    def fake_shared(n, group=None, device=None):
        assert n == 3 * _small().dim  # rows x dim floats per sum
        return lambda t, stream=None: seen.append(("sum", tuple(t.shape), stream))

    monkeypatch.setattr(C, "shared_peer_allreduce", fake_shared)
    cfg = _small()
    dec = M.LlamaDecoder(cfg, rows=3, device="cpu", weights=_weights(cfg, seed=9), group=object())
    monkeypatch.setattr(dec, "_gather_logits", lambda: seen.append(("gather",)))
    dec.step()
    assert seen == [("sum", (3, cfg.dim), dec.stream)] * (2 * cfg.n_layers) + [("gather",)]


@pytest.mark.parametrize("variant", ["bias", "qknorm"])
def test_qkv_extras_wiring(calls, tmp_path, variant):
    """Qwen-style files: after the q/k/v projections of every layer, one
    swq_qkv_bias_norm on the same rows (decode: rows; prefill: rows x P),
    with exactly the layer's biases / norms; Llama files never call it."""
    dec = M.LlamaDecoder.from_gguf(LG.write(tmp_path / "m.gguf", variant), rows=2, device="cpu")
    dec.step()
    ex = [c for c in calls if c[0] == "qkv_bias_norm"]
    assert len(ex) == dec.cfg.n_layers
    qd, kvd = dec.q_dim, dec.kv_dim
    for li, (_, a, kw) in enumerate(ex):
        L = dec.layers[li]
        assert a[0].data_ptr() == dec.qk.data_ptr() and a[1].data_ptr() == dec.qk.data_ptr() + 4 * qd
        assert a[2] is dec.v
        for i, key in enumerate(("bq", "bk", "bv", "q_norm", "k_norm")):
            assert a[3 + i] is L.get(key), key
        assert a[8:13] == (qd, kvd, dec.cfg.head_dim, dec.cfg.eps, 2)
        assert kw["ldq"] == kw["ldk"] == qd + kvd and kw["ldv"] == kvd
    names = [c[0] for c in calls]
    assert names.index("qkv_bias_norm") < names.index("rope_kv")
    calls.clear()
    dec.prefill([[1, 2, 3], [4, 5, 6]])
    ex = [c for c in calls if c[0] == "qkv_bias_norm"]
    assert len(ex) == dec.cfg.n_layers and all(c[1][12] == 6 for c in ex)


def test_llama_layers_never_call_qkv_extras(calls):
    cfg = _small()
    dec = M.LlamaDecoder(cfg, rows=1, device="cpu", weights=_weights(cfg, seed=9))
    dec.step()
    dec.prefill([[1, 2, 3]])
    assert not [c for c in calls if c[0] == "qkv_bias_norm"]


@pytest.mark.parametrize("rank", [0, 1])
def test_tensor_parallel_bias_slices(calls, monkeypatch, tmp_path, rank):
    """Each rank keeps the bias elements of its own heads; head norms whole."""
    import swq.parallel as P
    monkeypatch.setattr(P, "_world", lambda group: (rank, 2))
    from swq import gguf as G
    g = G.GGUFFile(LG.write(tmp_path / "b.gguf", "bias"))
    cfg = G.llama_config(g)
    W = G.llama_weights(g, cfg)
    dec = M.LlamaDecoder(cfg, rows=1, device="cpu", weights=W, group=object(), collective="nccl")
    for li, L in enumerate(dec.layers):
        for key, n in (("bq", dec.q_dim), ("bk", dec.kv_dim), ("bv", dec.kv_dim)):
            assert np.array_equal(L[key].numpy(), W["layers"][li][key][rank * n:(rank + 1) * n])


# ---------------------------------------------------------------- MoE decoder wiring
class _FakeMoE:
    """Records MoEFFN construction and calls (no device work)."""
    made = []

    def __init__(self, experts, types, H, F, router_w, top_k, max_tokens, **kw):
        self.args = dict(experts=experts, types=types, H=H, F=F, router=router_w, k=top_k, max_tokens=max_tokens, **kw)
        self.max_tokens = max_tokens
        self.calls = []
        _FakeMoE.made.append(self)

    def __call__(self, x, T, out=None, peer_tokens=None, stream=None):
        self.calls.append((x, T, out, peer_tokens))


def test_moe_decoder_wiring(calls, monkeypatch):
    import swq.moe
    from test_gpu_moe_model import _cfg, _weights
    _FakeMoE.made = []
    monkeypatch.setattr(swq.moe, "MoEFFN", _FakeMoE)
    cfg = _cfg()
    W = _weights(cfg, seed=2)
    dec = M.LlamaDecoder(cfg, rows=3, device="cpu", weights=W, moe_max_tokens=4)
    assert len(_FakeMoE.made) == cfg.n_layers
    first = _FakeMoE.made[0]
    for li, m in enumerate(_FakeMoE.made):
        a = m.args
        assert a["k"] == cfg.top_k and a["F"] == cfg.expert_ffn and a["max_tokens"] == 4
        assert a["scratch_from"] is (None if li == 0 else first)  # one set of buffers for all layers
        assert a["group"] is None and a["shared_F"] == cfg.shared_ffn
        assert len(a["experts"]) == cfg.n_experts
        np.testing.assert_array_equal(a["router"], W["layers"][li]["router"])
        e3 = np.asarray(W["layers"][li]["w_down_exps"]).reshape(cfg.n_experts, -1)[3]
        assert np.array_equal(a["experts"][3][2], e3)
    dec.step()
    g = _gemms(calls)
    # per layer: q|k, v, o -- no dense FFN projection -- then the LM head
    assert len(g) == 3 * cfg.n_layers + 1
    for li, m in enumerate(_FakeMoE.made):
        assert len(m.calls) == 1
        x, T, out, pt = m.calls[0]
        assert T == 3 and pt == 3 and out is dec.xb and x is dec.xn
    # prefill: rows x P = 3 x 3 = 9 rows in MoE calls of at most 4 rows
    for m in _FakeMoE.made:
        m.calls.clear()
    dec.prefill([[1, 2, 3], [4, 5, 6], [7, 8, 9]])
    for m in _FakeMoE.made:
        assert [c[1] for c in m.calls] == [4, 4, 1] and [c[3] for c in m.calls] == [4, 4, 1]
    with pytest.raises(ValueError):
        M.LlamaDecoder(cfg, rows=1, device="cpu", weights=W, group=object())


def test_ffn_split_keeps_down_rows_aligned():
    """The 70B shape's Q6_K w_down over 4 and 8 ranks: ffn / G columns are
    2940 or 5880 bytes per row, not a multiple of 16, so the FFN is split in
    units of 8 Q6_K blocks (2048 columns); over 2 ranks the even split is
    already aligned and stays."""
    cfg = M.LlamaConfig.llama3_70b()
    assert M.ffn_split(cfg, 2) == [(0, 14336), (14336, 14336)]
    assert M.ffn_split(cfg, 4) == [(0, 8192), (8192, 8192), (16384, 6144), (22528, 6144)]
    s8 = M.ffn_split(cfg, 8)
    assert [n for _, n in s8] == [4096] * 6 + [2048] * 2
    for G in (1, 2, 4, 8):
        parts = M.ffn_split(cfg, G)
        assert parts[0][0] == 0 and sum(n for _, n in parts) == cfg.ffn
        assert all(a + n == b for (a, n), (b, _) in zip(parts, parts[1:]))
        for _, n in parts:
            assert (n // 256 * 210) % 16 == 0
    # every layer's w_down type counts: Q4_K (512) with Q6_K (2048) -> 2048
    small = M.LlamaConfig(n_layers=2, dim=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=3 * 2048,
                          types=dict(M.LlamaConfig().types, w_down=synth.Q4_K))
    assert M.ffn_split(small, 4) == [(r * 1536, 1536) for r in range(4)]  # 1536 / 256 * 144 = 864 = 54 * 16


@pytest.mark.parametrize("rank", [0, 3])
def test_tensor_parallel_uneven_ffn_shards(calls, monkeypatch, rank):
    """An FFN of 14336 with a Q6_K w_down over 4 ranks: 3584 columns are not
    a whole 16-byte row unit, so the ranks take 4096, 4096, 4096 and 2048
    columns; rank r keeps exactly those gate/up rows and w_down columns and
    sizes its activation buffers to them."""
    import swq.parallel as P
    monkeypatch.setattr(P, "_world", lambda group: (rank, 4))
    cfg = M.LlamaConfig(n_layers=1, dim=256, n_heads=4, n_kv_heads=4, head_dim=64, ffn=14336, vocab=400,
                        max_seq=16)
    W = _weights_for(cfg, 11)
    dec = M.LlamaDecoder(cfg, rows=1, device="cpu", weights=W, group=object(), collective="nccl")
    f0, n = [(0, 4096), (4096, 4096), (8192, 4096), (12288, 2048)][rank]
    assert (dec.ffn_off, dec.ffn) == (f0, n)
    L, lt = dec.layers[0], cfg.layer_type_map(0)
    qk, bb = synth.block_geometry(lt["w_down"])
    down = W["layers"][0]["w_down"].reshape(cfg.dim, cfg.ffn // qk, bb)[:, f0 // qk:(f0 + n) // qk]
    assert np.array_equal(L["w_down"].numpy(), down.reshape(-1))
    qk, bb = synth.block_geometry(lt["w_gate"])
    gate = W["layers"][0]["w_gate"].reshape(cfg.ffn, -1)[f0:f0 + n]
    up = W["layers"][0]["w_up"].reshape(cfg.ffn, -1)[f0:f0 + n]
    if "w_gate_up" in L:
        ng = n * synth.row_bytes(lt["w_gate"], cfg.dim)
        assert np.array_equal(L["w_gate_up"][:ng].numpy(), gate.reshape(-1))
        assert np.array_equal(L["w_gate_up"][ng:].numpy(), up.reshape(-1))
    else:
        assert np.array_equal(L["w_gate"].numpy(), gate.reshape(-1))
    assert tuple(dec.h.shape) == (1, n) and tuple(dec.gu.shape) == (1, 2 * n)
