"""GGUF files: the on-disk format go-infer loads its weights from, read
without copying (mmap), and a writer (for tests, and to dump the seeded
synthetic models for other tools).

Reader — the format as go-infer parses it (pkg/gguf/gguf.go:20-48 OpenFile,
:146-240 parseHeader, :66-90 GetTensorData; constants pkg/gguf/types.go):
little-endian magic "GGUF", version 2 or 3, tensor count and key-value count
(u64), the key-value metadata (a length-prefixed key, a u32 value type, the
value; 13 value types, arrays of them), the tensor infos (name, u32 number
of dimensions, u64 dimensions in GGML order — dimension 0 is the row
length —, u32 GGML type, u64 offset into the data section), and the data
section at the next multiple of general.alignment (32 when absent).
Tensor byte sizes follow TensorByteSize (gguf.go:93-143).

Model configuration — the keys Engine reads (pkg/engine/engine.go:71-127):
<arch>.<suffix> first, then llama.<suffix>, then the default:
embedding_length, feed_forward_length, block_count, attention.head_count,
attention.head_count_kv (default head_count), context_length,
rope.freq_base (500000), attention.layer_norm_rms_epsilon (1e-5, then
attention.layer_norm_epsilon); the vocabulary size from the tokenizer
token list, else dimension 1 of token_embd.weight.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass

import numpy as np

MAGIC = 0x46554747  # "GGUF"
VERSIONS = (2, 3)

# metadata value types (types.go:9-21)
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

# GGML tensor types and their storage: (elements per block, bytes per block)
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K, GGML_BF16 = 0, 1, 2, 8, 12, 14, 29
_BLOCKS = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 9: (32, 40),
           10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292),
           16: (256, 66), 17: (256, 74), 18: (256, 98), 19: (256, 48), 20: (32, 18), 21: (256, 110),
           22: (256, 82), 23: (256, 136), 24: (1, 1), 25: (1, 2), 26: (1, 4), 27: (1, 8), 28: (1, 8), 29: (1, 2)}


def tensor_byte_size(ggml_type: int, n_elements: int) -> int:
    """Bytes of a tensor of n_elements (TensorByteSize, gguf.go:93-143;
    unknown types count 4 bytes per element, as there)."""
    per, nbytes = _BLOCKS.get(ggml_type, (1, 4))
    return (n_elements + per - 1) // per * nbytes


@dataclass
class TensorInfo:
    name: str
    dims: list  # GGML order: dims[0] is the row length
    type: int
    offset: int

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= int(d)
        return n if self.dims else 0


_MAX_DEPTH = 8  # nesting of metadata arrays
_MAX_DIMS = 4   # GGML tensors have at most four dimensions


def _min_size(vtype: int) -> int:
    """Fewest bytes a metadata value of this type occupies."""
    if vtype in _SCALAR:
        return struct.calcsize(_SCALAR[vtype])
    return {T_BOOL: 1, T_STR: 8, T_ARR: 12}.get(vtype, 1)


class _Cursor:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def room(self, count: int, each: int, what: str) -> None:
        """Refuse a count that cannot fit in the bytes left (a corrupted
        header would otherwise be parsed from the tensor data)."""
        if count * each > len(self.buf) - self.pos:
            raise ValueError(f"GGUF {what} count {count} exceeds the file")

    def take(self, fmt: str):
        size = struct.calcsize(fmt)
        if self.pos + size > len(self.buf):
            raise ValueError("GGUF header truncated")
        (v,) = struct.unpack_from(fmt, self.buf, self.pos)
        self.pos += size
        return v

    def string(self) -> str:
        n = self.take("<Q")
        if self.pos + n > len(self.buf):
            raise ValueError("GGUF header truncated")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8", errors="replace")
        self.pos += n
        return s

    def value(self, vtype: int, depth: int = 0):
        if vtype in _SCALAR:
            return self.take(_SCALAR[vtype])
        if vtype == T_BOOL:
            return self.take("<B") != 0
        if vtype == T_STR:
            return self.string()
        if vtype == T_ARR:
            if depth >= _MAX_DEPTH:
                raise ValueError("GGUF metadata arrays nested too deeply")
            etype, count = self.take("<I"), self.take("<Q")
            self.room(count, _min_size(etype), "array")
            return [self.value(etype, depth + 1) for _ in range(count)]
        raise ValueError(f"unsupported GGUF metadata type {vtype}")


class GGUFReader:
    """An opened GGUF file (gguf.Reader): .version, .metadata, .tensors
    (name -> TensorInfo), .data_offset; tensor bytes are views of the
    mapped file."""

    def __init__(self, path: str):
        self._file = open(path, "rb")
        try:
            self._map = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError:  # an empty file cannot be mapped
            self._file.close()
            raise ValueError("GGUF header truncated") from None
        try:
            self._parse()
        except Exception:
            self.close()
            raise

    def _parse(self) -> None:
        c = _Cursor(self._map)
        magic = c.take("<I")
        if magic != MAGIC:
            raise ValueError(f"invalid GGUF magic 0x{magic:08X}")
        self.version = c.take("<I")
        if self.version not in VERSIONS:
            raise ValueError(f"unsupported GGUF version {self.version}")
        n_tensors, n_kv = c.take("<Q"), c.take("<Q")
        c.room(n_kv, 8 + 4 + 1, "metadata")
        self.metadata = {}
        for _ in range(n_kv):
            key = c.string()
            self.metadata[key] = c.value(c.take("<I"))
        c.room(n_tensors, 8 + 4 + 4 + 8, "tensor")
        self.tensors = {}
        for _ in range(n_tensors):
            name = c.string()
            n_dims = c.take("<I")
            if n_dims > _MAX_DIMS:
                raise ValueError(f"tensor {name}: {n_dims} dimensions")
            dims = [c.take("<Q") for _ in range(n_dims)]
            self.tensors[name] = TensorInfo(name, dims, c.take("<I"), c.take("<Q"))
        align = self.metadata.get("general.alignment")
        align = align if isinstance(align, int) and align > 0 else 32
        self.data_offset = (c.pos + align - 1) // align * align

    def tensor_data(self, name: str) -> np.ndarray:
        """The tensor's raw bytes (GetTensorData): uint8, or float32 for F32."""
        info = self.tensors.get(name)
        if info is None:
            raise KeyError(f"tensor not found: {name}")
        start = self.data_offset + info.offset
        end = start + tensor_byte_size(info.type, info.n_elements)
        if start >= len(self._map) or end > len(self._map):
            raise ValueError(f"tensor {name} [{start}, {end}) exceeds the file ({len(self._map)} bytes)")
        raw = np.frombuffer(self._map, dtype=np.uint8, count=end - start, offset=start)
        return raw.view(np.float32) if info.type == GGML_F32 else raw

    # metadata helpers (GetMetadataUint / Float / String / Bool, gguf.go:318-392)
    def get_uint(self, key: str, default: int = 0) -> int:
        v = self.metadata.get(key)
        return int(v) if isinstance(v, int) and not isinstance(v, bool) else default

    def get_float(self, key: str, default: float = 0.0) -> float:
        v = self.metadata.get(key)
        return float(v) if isinstance(v, float) else default

    def get_string(self, key: str, default: str = "") -> str:
        v = self.metadata.get(key)
        return v if isinstance(v, str) else default

    def get_bool(self, key: str, default: bool = False) -> bool:
        v = self.metadata.get(key)
        if isinstance(v, bool):
            return v
        return v != 0 if isinstance(v, int) else default

    def close(self) -> None:
        if getattr(self, "_map", None) is not None:
            try:
                self._map.close()
            except BufferError:  # numpy views still alive: the map closes with them
                pass
            self._map = None
        if getattr(self, "_file", None) is not None:
            self._file.close()
            self._file = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


# ---- writer ------------------------------------------------------------------

@dataclass
class Typed:
    """A metadata value with an explicit GGUF value type (T_*); for arrays
    the value is (element type, list)."""
    vtype: int
    value: object


def _encode_value(out: bytearray, value, vtype: int) -> None:
    if vtype in _SCALAR:
        out += struct.pack(_SCALAR[vtype], value)
    elif vtype == T_BOOL:
        out += struct.pack("<B", 1 if value else 0)
    elif vtype == T_STR:
        b = value.encode("utf-8")
        out += struct.pack("<Q", len(b)) + b
    elif vtype == T_ARR:
        etype, items = value
        out += struct.pack("<IQ", etype, len(items))
        for it in items:
            _encode_value(out, it, etype)
    else:
        raise ValueError(f"unsupported GGUF metadata type {vtype}")


def _guess_type(value) -> tuple:
    if isinstance(value, bool):
        return T_BOOL, value
    if isinstance(value, int):
        return (T_U32, value) if 0 <= value < 2 ** 32 else (T_I64, value)
    if isinstance(value, float):
        return T_F32, value
    if isinstance(value, str):
        return T_STR, value
    if isinstance(value, (list, tuple)):  # homogeneous, typed by the first element; nested arrays too
        if not value:
            return T_ARR, (T_U32, [])
        et, _ = _guess_type(value[0])
        return T_ARR, (et, [_guess_type(v)[1] for v in value])
    raise TypeError(f"cannot store {type(value)} in GGUF metadata")


def write_gguf(path: str, metadata: dict, tensors: list, alignment: int = 32, version: int = 3) -> None:
    """Write a GGUF file.  metadata: key -> value (bool, int -> u32 or i64,
    float -> f32, str, list) or key -> Typed(vtype, value); tensors: (name,
    GGML type, dims in GGML order, bytes-like or array data)."""
    meta = dict(metadata)
    if alignment != 32:
        meta.setdefault("general.alignment", Typed(T_U32, alignment))
    out = bytearray(struct.pack("<IIQQ", MAGIC, version, len(tensors), len(meta)))
    for key, val in meta.items():
        vtype, v = (val.vtype, val.value) if isinstance(val, Typed) else _guess_type(val)
        _encode_value(out, key, T_STR)
        out += struct.pack("<I", vtype)
        _encode_value(out, v, vtype)
    offsets, blobs, off = [], [], 0
    for name, gtype, dims, data in tensors:
        blob = np.frombuffer(bytes(data), np.uint8) if isinstance(data, (bytes, bytearray)) else \
            np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        n = 1
        for d in dims:
            n *= int(d)
        if blob.size != tensor_byte_size(gtype, n):
            raise ValueError(f"{name}: {blob.size} bytes for {n} elements of type {gtype}")
        offsets.append(off)
        blobs.append(blob)
        off += (blob.size + alignment - 1) // alignment * alignment
    for (name, gtype, dims, _data), o in zip(tensors, offsets):
        _encode_value(out, name, T_STR)
        out += struct.pack("<I", len(dims))
        for d in dims:
            out += struct.pack("<Q", int(d))
        out += struct.pack("<IQ", gtype, o)
    out += b"\0" * ((-len(out)) % alignment)
    with open(path, "wb") as f:
        f.write(out)
        for blob in blobs:
            f.write(blob.tobytes())
            f.write(b"\0" * ((-blob.size) % alignment))


# ---- models ------------------------------------------------------------------

def model_config(reader: GGUFReader, max_seq: int = 8192):
    """synth.LlamaConfig from the metadata, with Engine's keys and defaults;
    max_seq caps the KV-cache length as the engine caps its active
    sequence length (8192)."""
    import synth

    arch = reader.get_string("general.architecture", "llama")

    def u(suffix, default):
        for key in (f"{arch}.{suffix}", f"llama.{suffix}"):
            v = reader.get_uint(key, 0)
            if v > 0:
                return v
        return default

    def f(suffix, default):
        for key in (f"{arch}.{suffix}", f"llama.{suffix}"):
            v = reader.get_float(key, 0.0)
            if v > 0:
                return v
        return default

    n_heads = u("attention.head_count", 32)
    eps = f("attention.layer_norm_rms_epsilon", 0.0) or f("attention.layer_norm_epsilon", 1e-5)
    vocab = len(reader.metadata.get("tokenizer.ggml.tokens", []) or [])
    if vocab == 0 and "token_embd.weight" in reader.tensors and len(reader.tensors["token_embd.weight"].dims) > 1:
        vocab = int(reader.tensors["token_embd.weight"].dims[1])
    seq = u("context_length", 2048)
    seq = min(seq if seq > 0 else max_seq, max_seq)
    return synth.LlamaConfig(n_layers=u("block_count", 16), dim=u("embedding_length", 2048),
                             hidden=u("feed_forward_length", 5632), n_heads=n_heads,
                             n_kv_heads=u("attention.head_count_kv", n_heads), vocab=vocab, max_seq=seq,
                             eps=float(np.float32(eps)), rope_theta=float(np.float32(f("rope.freq_base", 500000.0))))


def matrix_role(name: str):
    """Tensor-parallel role of a tensor (a key of synth.shard_slices): the
    layer matrices by their GGUF names, token_embd and output; the Q, K and
    V biases take their matrix's rows.  None for what every rank keeps
    whole (norms)."""
    import synth

    parts = name.split(".")
    if len(parts) == 4 and parts[0] == "blk":
        role = {v: k for k, v in synth.TENSOR_NAMES.items()}.get(parts[2])
        if parts[3] == "weight":
            return role
        if parts[3] == "bias" and role in ("wq", "wk", "wv"):
            return role
        return None
    return {"token_embd.weight": "token_embd", "output.weight": "output"}.get(name)


def shard_matrix(qtype: int, data: np.ndarray, rows: int, cols: int, r0: int, nr: int, c0: int, nc: int):
    """Rows [r0, r0 + nr) x columns [c0, c0 + nc) of a row-major GGUF matrix
    as contiguous raw blocks (uint8, or float32 for F32); the column range
    must fall on block boundaries."""
    per, nbytes = _BLOCKS[qtype]
    if cols % per or c0 % per or nc % per or not (0 <= r0 and r0 + nr <= rows and 0 <= c0 and c0 + nc <= cols):
        raise ValueError(f"shard rows [{r0}, {r0 + nr}) cols [{c0}, {c0 + nc}) of a {rows}x{cols} matrix "
                         f"of type {qtype} (blocks of {per})")
    rb = cols // per * nbytes
    raw = np.asarray(data).view(np.uint8).reshape(rows, rb)
    out = np.ascontiguousarray(raw[r0:r0 + nr, c0 // per * nbytes:(c0 + nc) // per * nbytes]).reshape(-1)
    return out.view(np.float32) if qtype == GGML_F32 else out


def host_model(reader: GGUFReader, max_seq: int = 8192, rank: int = 0, world: int = 1):
    """A synth.HostModel over the file's tensors.  world == 1: views of the
    mapped file (keep the reader open while they are used; DeviceModel
    copies them).  world > 1: rank's Megatron shard of every matrix
    (synth.shard_slices: rows of Q, K, V, gate, up and the output head with
    the Q/K/V biases, columns of the attention output and down projections;
    the token table and the norms whole) under the shard's configuration,
    as copies."""
    import synth

    cfg = model_config(reader, max_seq)
    if world <= 1:
        m = synth.HostModel(cfg)
        for name, info in reader.tensors.items():
            m.tensors[name] = (info.type, reader.tensor_data(name))
        return m
    sl = synth.shard_slices(cfg, rank, world)
    m = synth.HostModel(synth.shard_config(cfg, world))
    for name, info in reader.tensors.items():
        data = reader.tensor_data(name)
        role = matrix_role(name)
        if role is None:
            m.tensors[name] = (info.type, data.copy())
            continue
        r0, nr, c0, nc = sl[role]
        if name.endswith(".bias"):
            m.tensors[name] = (info.type, np.ascontiguousarray(data[r0:r0 + nr]))
            continue
        cols, rows = int(info.dims[0]), int(info.dims[1])
        m.tensors[name] = (info.type, shard_matrix(info.type, data, rows, cols, r0, nr, c0, nc))
    return m


def save_model(host, path: str) -> None:
    """Write a synth.HostModel as a GGUF file with llama.* metadata."""
    c = host.cfg
    meta = {"general.architecture": "llama", "llama.block_count": c.n_layers, "llama.embedding_length": c.dim,
            "llama.feed_forward_length": c.hidden, "llama.attention.head_count": c.n_heads,
            "llama.attention.head_count_kv": c.n_kv_heads, "llama.context_length": c.max_seq,
            "llama.rope.freq_base": float(c.rope_theta), "llama.attention.layer_norm_rms_epsilon": float(c.eps)}
    tensors = []
    for name, (qt, arr) in host.tensors.items():
        arr = np.asarray(arr)
        if qt == GGML_F32:
            dims = list(arr.shape[::-1]) if arr.ndim > 1 else [arr.size]
        else:
            rows = {"token_embd.weight": c.vocab, "output.weight": c.vocab}.get(name)
            if rows is None:
                import synth
                rows = synth.layer_shapes(c)[matrix_role(name)][0]
            per, nbytes = _BLOCKS[qt]
            cols = arr.size // rows // nbytes * per
            dims = [cols, rows]
        tensors.append((name, qt, dims, arr.view(np.uint8).reshape(-1)))
    write_gguf(path, meta, tensors)
