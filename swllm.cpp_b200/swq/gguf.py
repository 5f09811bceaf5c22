"""GGUF model files on the host side of libswq: read, write, and map a dense
Llama-family file onto LlamaDecoder.

Reading follows the reference's GGUFFile (src/gguf.h:224-419): the
little-endian magic 0x46554747 ("GGUF"), version 2 or 3, tensor and metadata
counts (u64), the metadata key/value pairs, the tensor infos (name, n_dims,
dims[n_dims], GGML type, offset), and the data section, which starts where the
header ends rounded up to ``general.alignment`` (32 when the key is absent).
A tensor's bytes start at data_offset + offset.  Metadata lookups keep the
reference's conversions (GGUFValue::to_int / to_float / to_string,
src/gguf.h:176-206): an integer read of a float, string or array value gives 0,
a float read of an integer gives its value, a string read of a non-string "".

Where the reference reads the whole file into a vector (src/gguf.h:238-257),
GGUFFile maps it read-only: a tensor is a view of the page cache until it is
uploaded to the GPU, so a multi-GB model is not copied on the host first.
Failures the reference prints and answers with ``false`` (no file, bad magic,
unsupported version, truncation) raise GGUFError.

``write_gguf`` writes the same format (version 3, every tensor's offset a
multiple of the alignment).  ``llama_from_gguf`` reads a dense Llama-family
file the way Model::load_config / load_weights do (src/model.h:586-689,
760-880) into a LlamaConfig and the weights dict LlamaDecoder takes, keeping
every projection in its GGUF blocks.
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass

import numpy as np

MAGIC = 0x46554747
DEFAULT_ALIGNMENT = 32

# GGMLType ids (src/gguf.h:18-40)
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q8_1 = 0, 1, 2, 3, 6, 7, 8, 9
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 10, 11, 12, 13, 14
I8, I16, I32, I64, F64, BF16, F8_E4M3, F8_E5M2 = 24, 25, 26, 27, 28, 30, 37, 38

# type -> (elements per block, bytes per block): ggml_block_size /
# ggml_type_size, src/gguf.h:60-118.  Unknown types have size 0, block 1.
GGML_TYPES = {
    F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22), Q5_1: (32, 24),
    Q8_0: (32, 34), Q8_1: (32, 40), Q2_K: (256, 84), Q3_K: (256, 110), Q4_K: (256, 144),
    Q5_K: (256, 176), Q6_K: (256, 210), I8: (1, 1), I16: (1, 2), I32: (1, 4), I64: (1, 8),
    F64: (1, 8), BF16: (1, 2), F8_E4M3: (1, 1), F8_E5M2: (1, 1),
}
# the formats libswq multiplies
QUANT_TYPES = (Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K)

# metadata value types (GGUFMetadataValueType, src/gguf.h:42-56)
(UINT8, INT8, UINT16, INT16, UINT32, INT32, FLOAT32, BOOL, STRING, ARRAY, UINT64, INT64,
 FLOAT64) = range(13)
_SCALAR = {UINT8: "<B", INT8: "<b", UINT16: "<H", INT16: "<h", UINT32: "<I", INT32: "<i",
           FLOAT32: "<f", BOOL: "<B", UINT64: "<Q", INT64: "<q", FLOAT64: "<d"}
_INTS = (UINT8, INT8, UINT16, INT16, UINT32, INT32, UINT64, INT64, BOOL)


def type_block(type_id: int) -> tuple[int, int]:
    """(elements per block, bytes per block) of a GGML type."""
    return GGML_TYPES.get(type_id, (1, 0))


class GGUFError(ValueError):
    pass


@dataclass
class GGUFValue:
    """One metadata value: its type, the value (int, float, bool, str, or a
    list of values for ARRAY) and, for arrays, the element type."""
    type: int
    value: object
    arr_type: int | None = None

    def to_int(self) -> int:
        """As an int64 (a UINT64 of 2^63 or more wraps, as the reference's cast)."""
        if self.type == BOOL:
            return 1 if self.value else 0
        if self.type == UINT64 and self.value >= 2 ** 63:
            return int(self.value) - 2 ** 64
        return int(self.value) if self.type in _INTS else 0

    def to_float(self) -> float:
        if self.type in (FLOAT32, FLOAT64):
            return float(self.value)
        return float(self.to_int())

    def to_string(self) -> str:
        return self.value if self.type == STRING else ""


@dataclass
class GGUFTensorInfo:
    """GGUFTensorInfo (src/gguf.h:212-230); dims padded with 1 to four."""
    name: str
    n_dims: int
    dims: tuple
    type: int
    offset: int

    def num_elements(self) -> int:
        n = 1
        for d in self.dims[:self.n_dims]:
            n *= d
        return n

    def num_bytes(self) -> int:
        bs, ts = type_block(self.type)
        return (self.num_elements() // bs) * ts


class GGUFFile:
    """A parsed GGUF file, memory-mapped read-only (``GGUFFile(path)``)."""

    def __init__(self, path: str | os.PathLike):
        self.path = str(path)
        try:
            with open(self.path, "rb") as f:
                self.file_size = os.fstat(f.fileno()).st_size
                self._map = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) if self.file_size else b""
        except OSError as e:
            raise GGUFError(f"cannot open file '{self.path}': {e}") from e
        self.version = 0
        self.tensor_count = 0
        self.metadata_kv_count = 0
        self.alignment = DEFAULT_ALIGNMENT
        self.data_offset = 0
        self.metadata: dict[str, GGUFValue] = {}
        self.tensors: dict[str, GGUFTensorInfo] = {}
        self._pos = 0
        self._parse()

    def close(self) -> None:
        if isinstance(self._map, mmap.mmap):
            try:
                self._map.close()
            except BufferError:  # arrays still view the mapping; it closes with them
                pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ------------------------------------------------------------ parsing
    def _take(self, n: int) -> int:
        p = self._pos
        if p + n > self.file_size:
            raise GGUFError(f"unexpected end of file in '{self.path}' at byte {p}")
        self._pos = p + n
        return p

    def _scalar(self, fmt: str):
        p = self._take(struct.calcsize(fmt))
        return struct.unpack_from(fmt, self._map, p)[0]

    def _string(self) -> str:
        n = self._scalar("<Q")
        p = self._take(n)
        return bytes(self._map[p:p + n]).decode("utf-8", errors="surrogateescape")

    def _value(self, vtype: int) -> GGUFValue:
        if vtype == STRING:
            return GGUFValue(STRING, self._string())
        if vtype == ARRAY:
            at = self._scalar("<I")
            n = self._scalar("<Q")
            if at in _SCALAR:  # numeric arrays in one read
                sz = struct.calcsize(_SCALAR[at])
                p = self._take(sz * n)
                vals = np.frombuffer(self._map, dtype=np.dtype(_SCALAR[at]), count=n, offset=p).tolist()
                if at == BOOL:
                    vals = [v != 0 for v in vals]
                return GGUFValue(ARRAY, [GGUFValue(at, v) for v in vals], at)
            return GGUFValue(ARRAY, [self._value(at) for _ in range(n)], at)
        if vtype not in _SCALAR:
            raise GGUFError(f"unknown metadata value type {vtype} in '{self.path}'")
        v = self._scalar(_SCALAR[vtype])
        return GGUFValue(vtype, v != 0 if vtype == BOOL else v)

    def _parse(self) -> None:
        magic = self._scalar("<I")
        if magic != MAGIC:
            raise GGUFError(f"not a GGUF file (magic: 0x{magic:08X})")
        self.version = self._scalar("<I")
        if self.version < 2 or self.version > 3:
            raise GGUFError(f"unsupported GGUF version {self.version}")
        self.tensor_count = self._scalar("<Q")
        self.metadata_kv_count = self._scalar("<Q")
        for _ in range(self.metadata_kv_count):
            key = self._string()
            val = self._value(self._scalar("<I"))
            if key == "general.alignment":
                self.alignment = val.to_int()
            self.metadata[key] = val
        for _ in range(self.tensor_count):
            name = self._string()
            n_dims = self._scalar("<I")
            if n_dims > 4:
                raise GGUFError(f"tensor '{name}' has {n_dims} dimensions (at most 4)")
            dims = tuple(self._scalar("<Q") for _ in range(n_dims)) + (1,) * (4 - n_dims)
            ttype = self._scalar("<I")
            offset = self._scalar("<Q")
            self.tensors[name] = GGUFTensorInfo(name, n_dims, dims, ttype, offset)
        self.data_offset = self._pos
        if self.alignment > 0:
            self.data_offset = (self.data_offset + self.alignment - 1) // self.alignment * self.alignment

    # ------------------------------------------------------------ lookups
    def has_metadata(self, key: str) -> bool:
        return key in self.metadata

    def get_i64(self, key: str, default: int = 0) -> int:
        v = self.metadata.get(key)
        return default if v is None else v.to_int()

    def get_f64(self, key: str, default: float = 0.0) -> float:
        v = self.metadata.get(key)
        return default if v is None else v.to_float()

    def get_str(self, key: str, default: str = "") -> str:
        v = self.metadata.get(key)
        return default if v is None else v.to_string()

    def get_i64_array(self, key: str) -> list[int]:
        v = self.metadata.get(key)
        if v is None or v.type != ARRAY:
            return []
        return [e.to_int() for e in v.value]

    def tensor_file_offset(self, name: str) -> int:
        return self.data_offset + self.tensors[name].offset

    def get_tensor_data(self, name: str) -> np.ndarray | None:
        """The tensor's bytes (uint8, read-only view of the mapping), or None."""
        info = self.tensors.get(name)
        if info is None:
            return None
        start, n = self.data_offset + info.offset, info.num_bytes()
        if start + n > self.file_size:
            raise GGUFError(f"tensor '{name}' runs past the end of '{self.path}'")
        return np.frombuffer(self._map, dtype=np.uint8, count=n, offset=start)

    def blocks(self, name: str) -> np.ndarray:
        """A matrix's GGUF blocks as [rows, row bytes] (dims[0] = K columns,
        dims[1] = N rows, src/model.h:729-758)."""
        info = self.tensors[name]
        bs, ts = type_block(info.type)
        K = info.dims[0]
        if ts == 0 or K == 0 or K % bs:
            raise GGUFError(f"tensor '{name}': type {info.type} rows of {K} elements are not whole blocks")
        return self.get_tensor_data(name).reshape(info.num_elements() // K, K // bs * ts)

    def float_array(self, name: str) -> np.ndarray:
        """An F32 / F16 / BF16 tensor as float32 (exact conversions)."""
        info = self.tensors[name]
        raw = self.get_tensor_data(name)
        if info.type == F32:
            return raw.view(np.float32)
        if info.type == F16:
            return raw.view(np.float16).astype(np.float32)
        if info.type == BF16:
            return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        raise GGUFError(f"tensor '{name}' has type {info.type}, not F32/F16/BF16")


# ---------------------------------------------------------------- writing

def _int_type(vals: list) -> int:
    if all(0 <= x < 2 ** 32 for x in vals):
        return UINT32
    if all(-2 ** 31 <= x < 2 ** 31 for x in vals):
        return INT32
    return INT64


def _infer(v) -> GGUFValue:
    if isinstance(v, GGUFValue):
        return v
    if isinstance(v, bool):
        return GGUFValue(BOOL, v)
    if isinstance(v, (int, np.integer)):
        return GGUFValue(_int_type([int(v)]), int(v))
    if isinstance(v, (float, np.floating)):
        return GGUFValue(FLOAT32, float(v))
    if isinstance(v, str):
        return GGUFValue(STRING, v)
    if isinstance(v, (list, tuple)):
        items = [_infer(e) for e in v]
        at = items[0].type if items else INT32
        if items and all(e.type in (UINT32, INT32, INT64) for e in items):  # one integer type for all
            at = _int_type([e.value for e in items])
            items = [GGUFValue(at, e.value) for e in items]
        if any(e.type != at for e in items):
            raise TypeError("a GGUF array holds values of one type")
        return GGUFValue(ARRAY, items, at)
    raise TypeError(f"no GGUF value type for {type(v).__name__}")


def _pack_value(out: list, val: GGUFValue, with_type: bool = True) -> None:
    if with_type:
        out.append(struct.pack("<I", val.type))
    if val.type == STRING:
        b = val.value.encode("utf-8", errors="surrogateescape")
        out.append(struct.pack("<Q", len(b)) + b)
    elif val.type == ARRAY:
        out.append(struct.pack("<IQ", val.arr_type, len(val.value)))
        for e in val.value:
            _pack_value(out, e if isinstance(e, GGUFValue) else GGUFValue(val.arr_type, e), False)
    else:
        out.append(struct.pack(_SCALAR[val.type], int(val.value) if val.type == BOOL else val.value))


def write_gguf(path: str | os.PathLike, metadata: dict, tensors: list, alignment: int = DEFAULT_ALIGNMENT) -> None:
    """Write a version-3 GGUF file.

    metadata: key -> GGUFValue, or a plain value (bool, int -> UINT32 /
    INT32 / INT64, float -> FLOAT32, str, list).  tensors: (name, GGML type,
    dims, data) with dims innermost first (dims[0] = row length) and data the
    tensor's bytes -- any array (its raw bytes are written), or a function
    that returns one, called when the tensor is written, so a model larger
    than memory can be written one tensor at a time.  A general.alignment
    entry other than `alignment` is rejected."""
    meta = {k: _infer(v) for k, v in metadata.items()}
    if "general.alignment" in meta and meta["general.alignment"].to_int() != alignment:
        raise ValueError("general.alignment disagrees with the alignment argument")
    out = [struct.pack("<IIQQ", MAGIC, 3, len(tensors), len(meta))]
    for k, v in meta.items():
        _pack_value(out, GGUFValue(STRING, k), False)
        _pack_value(out, v)
    offset, infos = 0, []
    for name, ttype, dims, _ in tensors:
        info = GGUFTensorInfo(name, len(dims), tuple(dims) + (1,) * (4 - len(dims)), ttype, offset)
        if type_block(ttype)[1] == 0:
            raise ValueError(f"tensor '{name}': unknown GGML type {ttype}")
        _pack_value(out, GGUFValue(STRING, name), False)
        out.append(struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims))
        out.append(struct.pack("<IQ", ttype, offset))
        infos.append(info)
        offset = (offset + info.num_bytes() + alignment - 1) // alignment * alignment
    header = b"".join(out)
    data_offset = (len(header) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(header)
        f.write(b"\0" * (data_offset - len(header)))
        pos = 0
        for info, (name, ttype, dims, data) in zip(infos, tensors):
            raw = np.ascontiguousarray(data() if callable(data) else data).view(np.uint8).reshape(-1)
            if raw.size != info.num_bytes():
                raise ValueError(f"tensor '{name}': {raw.size} bytes given, type {ttype} dims {dims} "
                                 f"need {info.num_bytes()}")
            f.write(b"\0" * (info.offset - pos))
            f.write(raw.data)
            pos = info.offset + raw.size


# ---------------------------------------------------------------- Llama models

# architectures whose RoPE rotates halves (neox) rather than adjacent pairs,
# src/model.h:629-634
NEOX_ARCHS = ("qwen2", "qwen3", "qwen2moe", "qwen35", "qwen35moe", "starcoder2", "phi3", "phi2", "gpt_neox",
              "stablelm", "codeshell")
_MATRICES = {"wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output", "w_gate": "ffn_gate",
             "w_up": "ffn_up", "w_down": "ffn_down"}
# GatedDeltaNet layers of hybrid (Qwen3.5) files, src/model.h:795-807: name in
# the weights dict -> GGUF stem of the projections (attn_qkv and ssm_out
# required, the others optional as the reference's), and of the F32 vectors
_LINEAR_MATRICES = {"w_qkv": "attn_qkv", "w_z": "attn_gate", "w_beta": "ssm_beta", "w_alpha": "ssm_alpha",
                    "w_dt": "ssm_dt", "w_ssm_out": "ssm_out"}
_LINEAR_VECTORS = {"ssm_a": "ssm_a", "conv1d": "ssm_conv1d.weight", "ssm_norm": "ssm_norm.weight"}
_FFN = ("w_gate", "w_up", "w_down")
# optional per-layer tensors the decoder applies after the q/k/v projections
# (src/model.h:291-318, loaded at :822-837): name in the weights dict -> GGUF stem
_EXTRAS = {"bq": "attn_q.bias", "bk": "attn_k.bias", "bv": "attn_v.bias", "q_norm": "attn_q_norm.weight",
           "k_norm": "attn_k_norm.weight"}


def llama_config(g: GGUFFile, context_override: int = 0):
    """LlamaConfig of a dense Llama-family GGUF, read as Model::load_config
    does (src/model.h:586-689): `{arch}.embedding_length` etc.; vocab from
    `{arch}.vocab_size`, else the token list's length; head_dim = hidden /
    heads unless `{arch}.attention.key_length` is set; context (the positions
    the KV cache holds) from `{arch}.context_length` (2048 when absent),
    lowered to context_override when that is smaller, or to 4096 when no
    override is given and the file's exceeds 8192; types from the file's
    tensors."""
    from .model import LlamaConfig
    arch = g.get_str("general.architecture", "llama")
    hidden = g.get_i64(f"{arch}.embedding_length", 0)
    layers = g.get_i64(f"{arch}.block_count", 0)
    heads = g.get_i64(f"{arch}.attention.head_count", 0)
    if hidden == 0 or layers == 0 or heads == 0:
        raise GGUFError(f"incomplete model config (hidden={hidden}, layers={layers}, heads={heads})")
    if arch == "qwen35moe":
        raise GGUFError(f"architecture '{arch}': hybrid MoE files are not supported by the decoder")
    vocab = g.get_i64(f"{arch}.vocab_size", g.get_i64("tokenizer.ggml.tokens", 0))
    if vocab == 0:
        tok = g.metadata.get("tokenizer.ggml.tokens")
        vocab = len(tok.value) if tok is not None and tok.type == ARRAY else 0
    head_dim = hidden // heads
    if g.get_i64(f"{arch}.attention.key_length", 0) > 0:
        head_dim = g.get_i64(f"{arch}.attention.key_length", 0)
    rope_dim = g.get_i64(f"{arch}.rope.dimension_count", 0)
    if rope_dim not in (0, head_dim):
        raise GGUFError(f"partial rotary embedding (rope dim {rope_dim} of head dim {head_dim}) is not supported")
    max_seq = g.get_i64(f"{arch}.context_length", 2048)
    if 0 < context_override < max_seq:  # Model::apply_context_override, src/model.h:944-954
        max_seq = context_override
    elif context_override == 0 and max_seq > 8192:
        max_seq = 4096
    # hybrid files: layer kinds from {arch}.attention.layer_types (0 full, 1
    # linear attention) and the GatedDeltaNet sizes with the reference's
    # defaults (src/model.h:637-678, :911-921)
    linear = ()
    lin = {}
    if arch == "qwen35":
        kinds = g.metadata.get(f"{arch}.attention.layer_types")
        kinds = [int(e.value) for e in kinds.value] if kinds is not None and kinds.type == ARRAY else []
        linear = tuple(li for li, k in enumerate(kinds[:layers]) if k != 0)
        n_kv = g.get_i64(f"{arch}.attention.head_count_kv", heads)
        lin = dict(lin_k_hd=g.get_i64(f"{arch}.attention.linear_key_length", 0) or head_dim,
                   lin_v_hd=g.get_i64(f"{arch}.attention.linear_value_length", 0) or head_dim,
                   lin_n_k=g.get_i64(f"{arch}.attention.linear_head_count_kv", 0) or heads,
                   lin_n_v=g.get_i64(f"{arch}.attention.linear_head_count", 0) or n_kv,
                   lin_conv=g.get_i64(f"{arch}.ssm.conv_kernel", 0) or 4)
    layer_types = []
    for li in range(layers):
        lt = {}
        if li in linear:
            for key, stem in _LINEAR_MATRICES.items():
                name = f"blk.{li}.{stem}.weight"
                if name in g.tensors:
                    lt[key] = g.tensors[name].type
                elif key in ("w_qkv", "w_ssm_out"):
                    raise GGUFError(f"tensor '{name}' not found (GatedDeltaNet layer {li})")
            stems = {k: _MATRICES[k] for k in _FFN}
        else:
            stems = _MATRICES
        for key, stem in stems.items():
            name = f"blk.{li}.{stem}.weight"
            if name not in g.tensors:
                raise GGUFError(f"tensor '{name}' not found")
            lt[key] = g.tensors[name].type
        layer_types.append(lt)
    out_name = "output.weight" if "output.weight" in g.tensors else "token_embd.weight"
    full = [lt for li, lt in enumerate(layer_types) if li not in linear]
    types = dict(full[0] if full else layer_types[0], output=g.tensors[out_name].type)
    stem_of = dict(_MATRICES, **_LINEAR_MATRICES)
    for name, t in [(f"blk.{li}.{stem_of[k]}.weight", t) for li, lt in enumerate(layer_types)
                    for k, t in lt.items()] + [(out_name, types["output"])]:
        if t not in QUANT_TYPES:
            raise GGUFError(f"tensor '{name}' has GGML type {t}; libswq multiplies "
                            f"Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K and Q6_K blocks")
    uniform = all(lt == layer_types[0] for lt in layer_types)
    return LlamaConfig(n_layers=layers, dim=hidden, n_heads=heads,
                       n_kv_heads=g.get_i64(f"{arch}.attention.head_count_kv", heads), head_dim=head_dim,
                       ffn=g.get_i64(f"{arch}.feed_forward_length", 0), vocab=vocab,
                       eps=float(np.float32(g.get_f64(f"{arch}.attention.layer_norm_rms_epsilon", 1e-5))),
                       theta=float(np.float32(g.get_f64(f"{arch}.rope.freq_base", 10000.0))),
                       rope_neox=arch in NEOX_ARCHS, max_seq=max_seq, types=types,
                       layer_types=None if uniform and not linear else tuple(layer_types),
                       linear_layers=linear, **lin)


def llama_weights(g: GGUFFile, cfg) -> dict:
    """The weights dict LlamaDecoder takes, as views of the mapped file:
    projections as [rows, row bytes] GGUF blocks, norms as float32, the
    embedding table as float32 (F32/F16/BF16) or as (type, blocks), which the
    decoder dequantizes on the device as the reference dequantizes it at load
    (src/model.h:771-772).  A file without output.weight ties the LM head to
    the embedding table (src/model.h:776-779); it must then be one of the
    quantized formats."""
    extra_len = {"bq": cfg.q_dim, "bk": cfg.kv_dim, "bv": cfg.kv_dim, "q_norm": cfg.head_dim,
                 "k_norm": cfg.head_dim}

    def check_shape(name, N, K):
        info = g.tensors.get(name)
        if info is None:
            raise GGUFError(f"tensor '{name}' not found")
        if info.n_dims != 2 or info.dims[0] != K or info.dims[1] != N:
            raise GGUFError(f"tensor '{name}' has dims {info.dims[:info.n_dims]}, expected ({K}, {N})")

    def vec(name, n):
        info = g.tensors.get(name)
        if info is None:
            raise GGUFError(f"tensor '{name}' not found")
        a = g.float_array(name)
        if a.size != n:
            raise GGUFError(f"tensor '{name}' has {a.size} elements, expected {n}")
        return a

    check_shape("token_embd.weight", cfg.vocab, cfg.dim)
    te_info = g.tensors["token_embd.weight"]
    if te_info.type in QUANT_TYPES:
        te_blocks = g.blocks("token_embd.weight")
        token_embd = (te_info.type, te_blocks)
    else:
        token_embd = g.float_array("token_embd.weight").reshape(cfg.vocab, cfg.dim)
    if "output.weight" in g.tensors:
        check_shape("output.weight", cfg.vocab, cfg.dim)
        output = g.blocks("output.weight")
    else:
        output = te_blocks  # quantized (checked by llama_config)
    layers = []
    for li in range(cfg.n_layers):
        # files that name the post-attention norm post_attention_norm
        # instead of ffn_norm: the reference's fallback, src/model.h:838-844
        ffn_norm = f"blk.{li}.ffn_norm.weight"
        if ffn_norm not in g.tensors and f"blk.{li}.post_attention_norm.weight" in g.tensors:
            ffn_norm = f"blk.{li}.post_attention_norm.weight"
        L = {"attn_norm": vec(f"blk.{li}.attn_norm.weight", cfg.dim), "ffn_norm": vec(ffn_norm, cfg.dim)}
        if li in cfg.linear_layers:
            lt = cfg.layer_type_map(li)
            for key, (N, K) in cfg.layer_shapes(li).items():
                if key in lt:
                    name = f"blk.{li}.{dict(_MATRICES, **_LINEAR_MATRICES)[key]}.weight"
                    check_shape(name, N, K)
                    L[key] = g.blocks(name)
            for key, stem in _LINEAR_VECTORS.items():
                name = f"blk.{li}.{stem}"
                if name in g.tensors:
                    n = {"ssm_a": cfg.lin_n_v, "conv1d": cfg.lin_value_dim * cfg.lin_conv,
                         "ssm_norm": cfg.lin_value_dim}[key]
                    L[key] = vec(name, n)
            layers.append(L)
            continue
        for key, (N, K) in cfg.shapes().items():
            name = f"blk.{li}.{_MATRICES[key]}.weight"
            check_shape(name, N, K)
            L[key] = g.blocks(name)
        for key, stem in _EXTRAS.items():
            if f"blk.{li}.{stem}" in g.tensors:
                L[key] = vec(f"blk.{li}.{stem}", extra_len[key])
        layers.append(L)
    return {"token_embd": token_embd, "output_norm": vec("output_norm.weight", cfg.dim), "output": output,
            "layers": layers}


def llama_from_gguf(path, context_override: int = 0):
    """(LlamaConfig, weights dict, GGUFFile) of a dense Llama-family GGUF file.
    The weights are views of the open file; keep the GGUFFile until they are
    uploaded (LlamaDecoder copies them to the device)."""
    g = GGUFFile(path)
    cfg = llama_config(g, context_override)
    return cfg, llama_weights(g, cfg), g
