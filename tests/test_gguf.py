"""GGUF files and the model-level oracle, on the CPU.

* swq.gguf's reader against the reference's GGUFFile (src/gguf.h, compiled
  from source): header, every tensor's info and data position, every metadata
  lookup with the reference's type conversions, rejection of broken files.
* swq.gguf.llama_config against the reference's Model::load_config
  (src/model.h:586-689, 944-954).
* The CPU restatement of the decode forward (oracle/model_ref.py), which the
  GPU decode tests compare against, pinned to the reference's own
  Model::forward: against golden logits the reference produced (committed,
  tests/golden/make_golden_model.py), and live where the reference builds.
"""
import struct

import numpy as np
import pytest

import llama_gguf as LG
from conftest import GOLDEN, rel_l2
from swq import gguf as G
from swq import synth
from swq.model import rope_freqs

# The restatement and the reference differ only in libm/numpy rounding of
# cos/sin/exp and the order of two short dot products: ~4e-7 measured.
FORWARD_TOL = 1e-5


def _model_ref():
    from oracle.ref_model import model_ref_available
    if not model_ref_available():
        pytest.skip("reference model library not built (needs the reference sources)")
    from oracle import ref_model
    return ref_model


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    d = tmp_path_factory.mktemp("gguf")
    return {v: LG.write(d / f"{v}.gguf", v) for v in LG.VARIANTS}


ALL_TYPES_META = {
    "u8": G.GGUFValue(G.UINT8, 200), "i8": G.GGUFValue(G.INT8, -100), "u16": G.GGUFValue(G.UINT16, 60000),
    "i16": G.GGUFValue(G.INT16, -30000), "u32": G.GGUFValue(G.UINT32, 4000000000),
    "i32": G.GGUFValue(G.INT32, -2000000000), "f32": G.GGUFValue(G.FLOAT32, 1.5),
    "bool_t": True, "bool_f": False, "str": "llama", "utf8": "größe ✓",
    "u64": G.GGUFValue(G.UINT64, 2 ** 63 + 5), "i64": G.GGUFValue(G.INT64, -(2 ** 40)),
    "f64": G.GGUFValue(G.FLOAT64, 2.0 ** -30), "arr_i": [3, 1, 4, 1, 5], "arr_neg": [-1, 2, -3],
    "arr_s": ["a", "bc", ""], "arr_f": [0.5, -0.25], "arr_nested": [[1, 2], [3]], "arr_empty": [],
    "empty_str": "",
}


def _write_all_types(path, alignment=32):
    tensors = [("a", G.F32, (3, 2), np.arange(6, dtype=np.float32)),
               ("b", G.Q4_K, (512, 3), synth.random_blocks(G.Q4_K, 3, 512, seed=1)),
               ("c", G.F16, (5,), np.arange(5, dtype=np.float16)),
               ("d", G.Q8_0, (64, 1, 2), synth.random_blocks(G.Q8_0, 2, 64, seed=2))]
    meta = dict(ALL_TYPES_META)
    if alignment != 32:
        meta["general.alignment"] = alignment
    G.write_gguf(path, meta, tensors, alignment=alignment)
    return tensors


@pytest.mark.parametrize("alignment", [32, 64, 256])
def test_write_read_roundtrip(tmp_path, alignment):
    p = tmp_path / "t.gguf"
    tensors = _write_all_types(p, alignment)
    g = G.GGUFFile(p)
    assert (g.version, g.tensor_count, g.alignment) == (3, 4, alignment)
    assert g.data_offset % alignment == 0
    for k, v in ALL_TYPES_META.items():
        got = g.metadata[k]
        want = G._infer(v)
        assert got.type == want.type, k
        if want.type == G.ARRAY:
            assert got.arr_type == want.arr_type, k
            flat = lambda a: [flat(e.value) if e.type == G.ARRAY else e.value for e in a]  # noqa: E731
            got_v, want_v = flat(got.value), flat(want.value)
            assert got_v == pytest.approx(want_v) if want.arr_type == G.FLOAT32 else got_v == want_v, k
        elif want.type == G.FLOAT32:
            assert got.value == np.float32(want.value), k
        else:
            assert got.value == want.value, k
    for name, t, dims, data in tensors:
        info = g.tensors[name]
        assert (info.type, info.n_dims, info.dims[:len(dims)]) == (t, len(dims), tuple(dims))
        assert info.offset % alignment == 0
        assert np.array_equal(g.get_tensor_data(name), np.ascontiguousarray(data).view(np.uint8).reshape(-1))
    assert np.array_equal(g.float_array("a"), np.arange(6, dtype=np.float32))
    assert np.array_equal(g.float_array("c"), np.arange(5, dtype=np.float32))
    assert g.blocks("b").shape == (3, 2 * 144)
    assert g.get_tensor_data("missing") is None


def test_lookup_conversions():
    """GGUFValue::to_int / to_float / to_string, src/gguf.h:176-206."""
    assert G.GGUFValue(G.FLOAT32, 2.5).to_int() == 0
    assert G.GGUFValue(G.STRING, "7").to_int() == 0
    assert G.GGUFValue(G.BOOL, True).to_int() == 1
    assert G.GGUFValue(G.INT16, -3).to_float() == -3.0
    assert G.GGUFValue(G.UINT32, 5).to_string() == ""


def _compare_with_reference(ref_model, path):
    g, r = G.GGUFFile(path), ref_model.RefGGUF(path)
    assert (g.version, g.tensor_count, g.metadata_kv_count, g.alignment, g.data_offset) == \
        (r.version, r.tensor_count, r.metadata_kv_count, r.alignment, r.data_offset)
    for name, t in g.tensors.items():
        assert r.tensor(name) == (t.type, t.n_dims, t.dims, t.offset, t.num_bytes(), g.tensor_file_offset(name)), name
    assert r.tensor("no.such.tensor") is None
    for key in list(g.metadata) + ["no.such.key"]:
        assert g.get_i64(key, -7) == r.get_i64(key, -7), key
        gf, rf = g.get_f64(key, -7.5), r.get_f64(key, -7.5)
        assert gf == rf or (np.isnan(gf) and np.isnan(rf)), key
        assert g.get_str(key) == r.get_str(key), key
        v = g.metadata.get(key)
        assert (len(v.value) if v is not None and v.type == G.ARRAY else -1) == r.array_len(key), key


def test_reader_matches_reference_gguffile(tmp_path, files):
    ref_model = _model_ref()
    p = tmp_path / "all.gguf"
    _write_all_types(p, 64)
    for path in [p, *files.values()]:
        _compare_with_reference(ref_model, path)


def test_broken_files_rejected(tmp_path, files):
    """Bad magic, unsupported versions, a header cut short: GGUFError here,
    a failed load in the reference."""
    good = files["mix"].read_bytes()
    gm = G.GGUFFile(files["mix"])
    hdr_end = gm.data_offset - gm.alignment  # inside the header (before its padding)
    cases = {"magic": b"GGUG" + good[4:], "v1": good[:4] + struct.pack("<I", 1) + good[8:],
             "v4": good[:4] + struct.pack("<I", 4) + good[8:], "empty": b""}
    for cut in (3, 10, 30, hdr_end // 2, hdr_end - 1):
        cases[f"cut{cut}"] = good[:cut]
    from oracle.ref_model import model_ref_available
    for name, blob in cases.items():
        p = tmp_path / f"{name}.gguf"
        p.write_bytes(blob)
        with pytest.raises(G.GGUFError):
            G.GGUFFile(p)
        if model_ref_available():
            from oracle.ref_model import RefGGUF
            with pytest.raises(ValueError):
                RefGGUF(p)
    with pytest.raises(G.GGUFError):
        G.GGUFFile(tmp_path / "does-not-exist.gguf")
    # data cut short: the header parses, the tensor's bytes are missing
    p = tmp_path / "short_data.gguf"
    p.write_bytes(good[:-100])
    g = G.GGUFFile(p)
    last = max(g.tensors.values(), key=lambda t: t.offset)
    with pytest.raises(G.GGUFError):
        g.get_tensor_data(last.name)


@pytest.mark.parametrize("variant", list(LG.VARIANTS))
def test_golden_files_rebuild_identically(tmp_path, variant):
    gold = np.load(GOLDEN / f"golden_llama_{variant}.npz")
    assert LG.sha256(LG.write(tmp_path / "m.gguf", variant)) == str(gold["sha256"])


@pytest.mark.parametrize("variant", list(LG.VARIANTS))
def test_llama_config_matches_reference(files, variant):
    gold = np.load(GOLDEN / f"golden_llama_{variant}.npz")
    cfg = G.llama_config(G.GGUFFile(files[variant]))
    c = dict(zip(("hidden", "ffn", "layers", "heads", "kv_heads", "head_dim", "vocab", "max_seq", "rope_neox",
                  "rope_dim"), gold["config"].tolist()))
    assert (cfg.dim, cfg.ffn, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.vocab, cfg.max_seq,
            int(cfg.rope_neox)) == (c["hidden"], c["ffn"], c["layers"], c["heads"], c["kv_heads"], c["head_dim"],
                                    c["vocab"], c["max_seq"], c["rope_neox"])
    assert c["rope_dim"] == cfg.head_dim
    assert np.float32(cfg.eps) == gold["config_f"][0] and np.float32(cfg.theta) == gold["config_f"][1]
    want = LG.VARIANTS[variant]["layers"]
    assert [cfg.layer_type_map(li) for li in range(cfg.n_layers)] == want


@pytest.mark.parametrize("override", [0, 8, 31, 32, 100])
def test_context_override_as_reference(tmp_path, files, override):
    """Model::apply_context_override (src/model.h:944-954): an override only
    lowers the context; none given caps a context above 8192 at 4096."""
    assert G.llama_config(G.GGUFFile(files["mix"]), override).max_seq == (override if 0 < override < 32 else 32)
    ref_model = _model_ref()
    assert ref_model.RefModel(files["mix"], override).config["max_seq"] == \
        G.llama_config(G.GGUFFile(files["mix"]), override).max_seq


def test_long_context_capped_without_override(tmp_path):
    g = G.GGUFFile(files_with(tmp_path, {"llama.context_length": 131072}))
    assert G.llama_config(g).max_seq == 4096
    assert G.llama_config(g, 16384).max_seq == 16384


def files_with(tmp_path, changes: dict, drop=(), extra_tensors=(), retype=None):
    """The "tied" model rewritten with metadata changes, tensors dropped or
    added, or one tensor's GGML type changed."""
    src = G.GGUFFile(LG.write(tmp_path / "base.gguf", "tied"))
    meta = {k: v for k, v in src.metadata.items()}
    meta.update({k: v for k, v in changes.items()})
    tensors = []
    for name, info in src.tensors.items():
        if name in drop:
            continue
        data, t = src.get_tensor_data(name), info.type
        if retype and name == retype[0]:
            t = retype[1]
            data = np.zeros(G.GGUFTensorInfo(name, info.n_dims, info.dims, t, 0).num_bytes(), np.uint8)
        tensors.append((name, t, info.dims[:info.n_dims], data))
    tensors += list(extra_tensors)
    p = tmp_path / f"m{len(list(tmp_path.iterdir()))}.gguf"
    G.write_gguf(p, meta, tensors, alignment=src.alignment)
    return p


def test_unsupported_models_rejected(tmp_path):
    for kw in (dict(changes={"general.architecture": "qwen35moe"}),
               dict(changes={"llama.rope.dimension_count": 32}),
               dict(changes={}, drop=("blk.1.ffn_up.weight",)),
               dict(changes={}, retype=("blk.0.attn_q.weight", G.F16)),
               dict(changes={"llama.block_count": 0})):
        p = files_with(tmp_path, **kw)
        with pytest.raises(G.GGUFError):
            cfg = G.llama_config(G.GGUFFile(p))
            G.llama_weights(G.GGUFFile(p), cfg)


def test_hybrid_file_without_its_linear_projections_rejected(tmp_path):
    """A GatedDeltaNet layer needs attn_qkv and ssm_out (the reference runs
    such a layer as an identity residual, src/model.h:508; the decoder
    refuses the file instead)."""
    src = G.GGUFFile(LG.write(tmp_path / "h.gguf", "hybrid"))
    for drop in ("blk.0.attn_qkv.weight", "blk.0.ssm_out.weight"):
        tensors = [(n, i.type, i.dims[:i.n_dims], src.get_tensor_data(n)) for n, i in src.tensors.items() if n != drop]
        p = tmp_path / f"d{len(list(tmp_path.iterdir()))}.gguf"
        G.write_gguf(p, dict(src.metadata), tensors, alignment=src.alignment)
        with pytest.raises(G.GGUFError):
            G.llama_config(G.GGUFFile(p))


def test_neox_architectures(tmp_path):
    a = "qwen2"
    meta = {k.replace("llama.", f"{a}."): v for k, v in G.GGUFFile(LG.write(tmp_path / "b.gguf", "tied")).metadata.items()}
    meta["general.architecture"] = a
    p = files_with(tmp_path, meta)
    assert G.llama_config(G.GGUFFile(p)).rope_neox


def test_weights_are_views_of_the_file(files):
    """Projections are views of the mapped file: nothing is copied on the host
    before the upload."""
    cfg, W, g = G.llama_from_gguf(files["mix"])
    for key in ("wq", "w_down"):
        a = W["layers"][1][key]
        assert not a.flags.writeable and not a.flags.owndata
        name = f"blk.1.{LG._STEMS[key]}.weight"
        assert np.array_equal(a.reshape(-1), g.get_tensor_data(name))
    assert isinstance(W["token_embd"], np.ndarray) and W["token_embd"].shape == (cfg.vocab, cfg.dim)
    cfg2, W2, _ = G.llama_from_gguf(files["tied"])
    assert isinstance(W2["token_embd"], tuple) and W2["token_embd"][0] == G.Q8_0
    assert W2["output"] is W2["token_embd"][1] and cfg2.types["output"] == G.Q8_0


@pytest.mark.parametrize("variant", list(LG.VARIANTS))
def test_restated_forward_matches_reference_golden(files, variant):
    """oracle/model_ref.py's forward against the logits the reference's own
    Model::forward produced for the same file and tokens."""
    from oracle.model_ref import RefLlama
    gold = np.load(GOLDEN / f"golden_llama_{variant}.npz")
    cfg, W, _ = G.llama_from_gguf(files[variant])
    ref = RefLlama(cfg, W, rope_freqs(cfg), cfg.max_seq)
    for pos, tok in enumerate(gold["tokens"].tolist()):
        got = ref.forward(tok, pos)
        want = gold["logits"][pos]
        assert rel_l2(got, want) <= FORWARD_TOL, (pos, rel_l2(got, want))
        assert int(np.argmax(got)) == int(np.argmax(want))


@pytest.mark.parametrize("variant", list(LG.VARIANTS))
def test_restated_forward_matches_reference_live(files, variant):
    ref_model = _model_ref()
    from oracle.model_ref import RefLlama
    cfg, W, _ = G.llama_from_gguf(files[variant])
    m = ref_model.RefModel(files[variant])
    ref = RefLlama(cfg, W, rope_freqs(cfg), cfg.max_seq)
    toks = [3, 250, 17, 17, 88, 1, 299, 42]
    for pos, tok in enumerate(toks):
        assert rel_l2(ref.forward(tok, pos), m.forward(tok, pos)) <= FORWARD_TOL, pos


@pytest.mark.parametrize("ttype", [G.F32, G.F16, G.BF16])
def test_float_tables_as_reference_dequantize(tmp_path, ttype):
    """F32 / F16 / BF16 norm and embedding tables read as the reference's
    dequantize() reads them at load (src/tensor.h:451-460): bit for bit,
    subnormals, infinities and signed zeros included."""
    from oracle import ref_available, ref_dequantize
    bits = np.random.default_rng(3).integers(0, 2 ** 16, size=4096, dtype=np.uint16)
    bits[:6] = [0x0000, 0x8000, 0x0001, 0x7C00, 0xFC00, 0x03FF]
    data = np.random.default_rng(4).standard_normal(4096).astype(np.float32) if ttype == G.F32 else bits
    p = tmp_path / "f.gguf"
    G.write_gguf(p, {"general.architecture": "llama"}, [("t", ttype, (data.size,), data)])
    got = G.GGUFFile(p).float_array("t")
    if ttype == G.F32:
        assert np.array_equal(got.view(np.uint32), data.view(np.uint32))
    if ref_available():
        want = ref_dequantize(ttype, data.view(np.uint8), data.size)
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan)
        assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


def test_tensor_ranks_and_writer_errors(tmp_path):
    p = tmp_path / "r.gguf"
    t3 = np.arange(24, dtype=np.float32)
    t4 = synth.random_blocks(G.Q8_0, 4, 64, seed=5)
    G.write_gguf(p, {}, [("three", G.F32, (2, 3, 4), t3), ("four", G.Q8_0, (64, 2, 1, 2), t4)])
    g = G.GGUFFile(p)
    assert g.tensors["three"].dims == (2, 3, 4, 1) and g.tensors["three"].num_elements() == 24
    assert g.tensors["four"].num_bytes() == t4.nbytes and g.blocks("four").shape == (4, 68)
    with pytest.raises(ValueError):  # bytes do not match the type and dims
        G.write_gguf(tmp_path / "e1.gguf", {}, [("x", G.F32, (5,), np.zeros(4, np.float32))])
    with pytest.raises(ValueError):  # no such GGML type
        G.write_gguf(tmp_path / "e2.gguf", {}, [("x", 99, (4,), np.zeros(4, np.uint8))])
    with pytest.raises(ValueError):
        G.write_gguf(tmp_path / "e3.gguf", {"general.alignment": 64}, [], alignment=32)
    with pytest.raises(TypeError):  # mixed array element types
        G.write_gguf(tmp_path / "e4.gguf", {"a": [1, "x"]}, [])
    with pytest.raises(G.GGUFError):  # rows not whole blocks
        G.write_gguf(tmp_path / "e5.gguf", {}, [("q", G.Q4_K, (100, 1), np.zeros(0, np.uint8))])
        G.GGUFFile(tmp_path / "e5.gguf").blocks("q")


def _random_gguf(rng, path):
    """A random, valid GGUF file: every metadata value type (nested arrays
    too), tensors of every GGML type and rank 1-4, an uncommon alignment."""
    scalar_types = [G.UINT8, G.INT8, G.UINT16, G.INT16, G.UINT32, G.INT32, G.FLOAT32, G.BOOL, G.UINT64, G.INT64,
                    G.FLOAT64]
    lims = {G.UINT8: (0, 255), G.INT8: (-128, 127), G.UINT16: (0, 65535), G.INT16: (-32768, 32767),
            G.UINT32: (0, 2 ** 32 - 1), G.INT32: (-2 ** 31, 2 ** 31 - 1), G.UINT64: (0, 2 ** 64 - 1),
            G.INT64: (-2 ** 63, 2 ** 63 - 1)}

    def value(t):
        if t in lims:
            lo, hi = lims[t]
            return G.GGUFValue(t, int(rng.integers(lo, hi, endpoint=True, dtype=np.uint64 if t == G.UINT64
                                                   else np.int64)))
        if t == G.BOOL:
            return G.GGUFValue(t, bool(rng.integers(0, 2)))
        if t in (G.FLOAT32, G.FLOAT64):
            return G.GGUFValue(t, float(np.float32(rng.standard_normal())) if t == G.FLOAT32
                               else float(rng.standard_normal()))
        return G.GGUFValue(G.STRING, "".join(chr(int(c)) for c in rng.integers(32, 0x2FF, size=rng.integers(0, 12))))

    meta = {}
    for i in range(int(rng.integers(1, 25))):
        kind = rng.integers(0, 4)
        if kind == 0:
            v = value(G.STRING)
        elif kind == 1:
            v = value(scalar_types[rng.integers(len(scalar_types))])
        elif kind == 2:
            t = [G.STRING, *scalar_types][rng.integers(len(scalar_types) + 1)]
            v = G.GGUFValue(G.ARRAY, [value(t) for _ in range(rng.integers(0, 6))], t)
        else:
            inner = scalar_types[rng.integers(len(scalar_types))]
            v = G.GGUFValue(G.ARRAY, [G.GGUFValue(G.ARRAY, [value(inner) for _ in range(rng.integers(0, 3))], inner)
                                      for _ in range(rng.integers(0, 3))], G.ARRAY)
        meta[f"k{i}.{rng.integers(1000)}"] = v
    alignment = int([8, 16, 32, 64, 128][rng.integers(5)])
    meta["general.alignment"] = G.GGUFValue(G.UINT32, alignment)
    tensors = []
    for i in range(int(rng.integers(0, 8))):
        t = list(G.GGML_TYPES)[rng.integers(len(G.GGML_TYPES))]
        bs, ts = G.type_block(t)
        rank = int(rng.integers(1, 5))
        dims = [int(bs * rng.integers(1, 4))] + [int(rng.integers(1, 4)) for _ in range(rank - 1)]
        n = int(np.prod(dims)) // bs * ts
        tensors.append((f"t{i}", t, tuple(dims), rng.integers(0, 256, size=n, dtype=np.uint8)))
    G.write_gguf(path, meta, tensors, alignment=alignment)


@pytest.mark.parametrize("seed", range(12))
def test_random_files_read_as_reference(tmp_path, seed):
    ref_model = _model_ref()
    p = tmp_path / f"r{seed}.gguf"
    _random_gguf(np.random.default_rng(1000 + seed), p)
    _compare_with_reference(ref_model, p)
    g = G.GGUFFile(p)
    for name, info in g.tensors.items():  # and the bytes are where both say they are
        raw = p.read_bytes()
        off = g.tensor_file_offset(name)
        assert np.array_equal(g.get_tensor_data(name), np.frombuffer(raw[off:off + info.num_bytes()], np.uint8))


def test_minimal_header_as_reference_test(tmp_path):
    """The reference's tests/test_gguf.cpp:199-243 builds a GGUF v3 header with
    no metadata and no tensors: magic 0x46554747 ("GGUF"), version 3, two
    zero u64 counts.  The writer emits exactly those 24 bytes for an empty
    file; the reader (and the reference's) parse it, the data section at 32."""
    p = tmp_path / "min.gguf"
    G.write_gguf(p, {}, [])
    raw = p.read_bytes()
    assert raw[:4] == b"GGUF" and raw[:24] == struct.pack("<IIQQ", 0x46554747, 3, 0, 0)
    g = G.GGUFFile(p)
    assert (g.version, g.tensor_count, g.metadata_kv_count, g.data_offset) == (3, 0, 0, 32)
    p24 = tmp_path / "min24.gguf"
    p24.write_bytes(raw[:24])  # the reference test's buffer, no padding
    g24 = G.GGUFFile(p24)
    assert (g24.version, g24.tensors, g24.metadata) == (3, {}, {})
    from oracle.ref_model import model_ref_available
    if model_ref_available():
        from oracle.ref_model import RefGGUF
        r = RefGGUF(p24)
        assert (r.version, r.tensor_count, r.metadata_kv_count, r.data_offset) == (3, 0, 0, 32)


def test_context_cap_known_answers(tmp_path):
    """The reference's test_context_auto_cap (tests/test_gguf.cpp:1040-1072):
    40960 -> 4096 without an override, 4096 unchanged, an explicit 2048 kept."""
    g = G.GGUFFile(files_with(tmp_path, {"llama.context_length": 40960}))
    assert G.llama_config(g).max_seq == 4096 and G.llama_config(g, 2048).max_seq == 2048
    g = G.GGUFFile(files_with(tmp_path, {"llama.context_length": 4096}))
    assert G.llama_config(g).max_seq == 4096


def test_qwen3_architecture_config(tmp_path):
    """The reference's test_qwen3_config (tests/test_gguf.cpp:727-760): qwen3
    runs neox RoPE, head_dim = hidden / heads."""
    src = G.GGUFFile(LG.write(tmp_path / "b.gguf", "tied"))
    meta = {k.replace("llama.", "qwen3."): v for k, v in src.metadata.items()}
    meta["general.architecture"] = "qwen3"
    cfg = G.llama_config(G.GGUFFile(files_with(tmp_path, meta)))
    assert cfg.rope_neox and cfg.head_dim == cfg.dim // cfg.n_heads


def test_post_attention_norm_fallback(tmp_path):
    """Without ffn_norm.weight the post-attention norm is read from
    post_attention_norm.weight, as the reference's load_weights does
    (src/model.h:838-844, tests/test_gguf.cpp:1358-1398)."""
    src = G.GGUFFile(LG.write(tmp_path / "b.gguf", "tied"))
    norm = src.float_array("blk.1.ffn_norm.weight").copy()
    p = files_with(tmp_path, {}, drop=("blk.1.ffn_norm.weight",),
                   extra_tensors=[("blk.1.post_attention_norm.weight", G.F32, (norm.size,), norm)])
    g = G.GGUFFile(p)
    W = G.llama_weights(g, G.llama_config(g))
    assert np.array_equal(W["layers"][1]["ffn_norm"], norm)
    p2 = files_with(tmp_path, {}, drop=("blk.1.ffn_norm.weight",))
    with pytest.raises(G.GGUFError):
        g2 = G.GGUFFile(p2)
        G.llama_weights(g2, G.llama_config(g2))


def test_restated_rope_known_answers():
    """The reference's test_cpu_rope / _gqa / _neox (tests/test_gguf.cpp:508-600)
    on the restatement's two RoPE functions: identity at position 0; at
    position 1 a unit vector turns by angle 1 (freq 1/theta^0) into
    (cos 1, sin 1), on the next element (interleaved) or the one head_dim/2
    away (neox), alike in every head (GQA)."""
    from oracle.model_ref import rope_interleaved, rope_neox
    freqs = (1.0 / np.power(np.float32(10000.0), np.arange(2, dtype=np.float32) * 2 / np.float32(4))).astype(
        np.float32)
    c, s = np.cos(np.float32(1.0)), np.sin(np.float32(1.0))
    for rope in (rope_interleaved, rope_neox):
        v = np.array([1, 2, 3, 4, 5, 6, 7, 8], np.float32)
        assert np.allclose(rope(v, 4, 0, freqs), v, atol=1e-5)
    q = np.array([1, 0, 0, 0, 1, 0, 0, 0], np.float32)
    out = rope_interleaved(q, 4, 1, freqs)
    assert np.allclose(out[[0, 1, 4, 5]], [c, s, c, s], atol=1e-5)
    out = rope_neox(q, 4, 1, freqs)
    assert np.allclose(out[[0, 2, 4, 6]], [c, s, c, s], atol=1e-5)


def test_restated_elementwise_known_answers():
    """The reference's test_cpu_rmsnorm / _softmax (tests/test_gguf.cpp) on
    the restatement's RMSNorm and softmax."""
    from oracle.model_ref import rmsnorm, softmax
    x = np.array([1, 2, 3, 4], np.float32)
    rms = np.sqrt(np.float32(30 / 4) + np.float32(1e-5))
    assert np.allclose(rmsnorm(x, np.ones(4, np.float32), 1e-5), x / rms, atol=1e-4)
    e = np.exp(np.array([1, 2, 3], np.float64))
    sm = softmax(np.array([1, 2, 3], np.float32))
    assert abs(float(sm.sum()) - 1.0) < 1e-5 and np.allclose(sm, e / e.sum(), atol=1e-5)
