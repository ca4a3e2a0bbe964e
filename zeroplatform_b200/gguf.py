"""GGUF model files -> the device engine, zero-copy from the page cache.

Restates ZeroLlm's GGUF reader and loader:
* `GgufFile` = GgufReader.Read (ZeroLlm/src/ZeroLlm.Core/Format/GgufReader.cs:40-95: magic 'GGUF', versions 2 and
  3, tensor and metadata counts, typed metadata values including arrays, tensor infos, the data section aligned to
  `general.alignment`) over a read-only memory map, with GgufMemoryMappedReader.GetTensorBytes
  (Format/GgufMemoryMappedReader.cs:43-56: payload at data offset + tensor offset, bounds-checked) and
  GgufTensorInfo.GetSizeInBytes (Format/GgufTensorInfo.cs:43-67).
* `model_from_gguf` = LlmModel.LoadGguf (Engine/LlmModel.cs:270-466): the `{arch}.*` hyper-parameters with the
  reference's defaults (a key counts only when it holds the type the reference asks for, as
  GgufMetadata.TryGet<T> does), embedding width and vocabulary from `token_embd.weight`'s dimensions, the
  `blk.{l}.*` tensor names, and the LM head tied to the token embeddings when `output.weight` is absent.
* `write_gguf` = GgufWriter.WriteTo (Format/GgufWriter.cs:34-96): v3, every tensor padded to the alignment;
  `save_gguf` = LlmModel.SaveGguf (Engine/LlmModel.cs:167-264) for dense Q8_0 models: the same metadata keys and
  tensor names, dimensions [in, out].
`load_engine` hands the mapped Q8_0 tensors straight to zcu_engine_set_weight (one host -> device copy per tensor,
no intermediate buffer).
"""
from __future__ import annotations

import mmap
import struct

import numpy as np

GGUF_MAGIC = 0x46554747  # 'GGUF' little-endian

# GgufMetadataValueType (Format/GgufTypes.cs:6-21)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", U64: "<Q", I64: "<q",
           F64: "<d"}

# GgufTensorType (Format/GgufTypes.cs:26-56), the ones the size rule distinguishes
T_F32, T_F16, T_Q4_0, T_Q8_0 = 0, 1, 2, 8
T_I8, T_I16, T_I32, T_I64, T_F64, T_BF16 = 24, 25, 26, 27, 28, 29


class Typed:
    """A metadata value with the GGUF type it was stored as (the reference's typed lookups depend on it)."""
    __slots__ = ("type", "value")

    def __init__(self, vtype: int, value):
        self.type, self.value = vtype, value

    def __repr__(self):
        return f"Typed({self.type}, {self.value!r})"


class TensorInfo:
    def __init__(self, name: str, dims: list[int], ttype: int, offset: int):
        self.name, self.dims, self.type, self.offset = name, dims, ttype, offset

    @property
    def element_count(self) -> int:
        if not self.dims:
            return 0
        n = 1
        for d in self.dims:
            n *= d
        return n

    def size_in_bytes(self) -> int:
        """GgufTensorInfo.GetSizeInBytes: unknown types fall back to 4 bytes an element, as the reference does."""
        n = self.element_count
        if self.type in (T_F32, T_I32):
            return n * 4
        if self.type in (T_F16, T_BF16, T_I16):
            return n * 2
        if self.type in (T_F64, T_I64):
            return n * 8
        if self.type == T_I8:
            return n
        if self.type == T_Q8_0:
            return n // 32 * 34
        if self.type == T_Q4_0:
            return n // 32 * 18
        return n * 4


class _Cursor:
    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, fmt: str):
        v = struct.unpack_from(fmt, self.buf, self.pos)[0]
        self.pos += struct.calcsize(fmt)
        return v

    def string(self) -> str:
        n = self.take("<Q")
        if n > 0x7FFFFFFF:
            raise ValueError("String length exceeds Int32.MaxValue.")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8")
        self.pos += n
        return s

    def value(self, vtype: int):
        if vtype in _SCALAR:
            return self.take(_SCALAR[vtype])
        if vtype == BOOL:
            return self.take("<B") != 0
        if vtype == STRING:
            return self.string()
        if vtype == ARRAY:
            et = self.take("<I")
            n = self.take("<Q")
            if n > 0x7FFFFFFF:
                raise ValueError("Array element count exceeds Int32.MaxValue.")
            return [Typed(et, self.value(et)) for _ in range(n)]
        raise ValueError(f"Unknown GGUF metadata type: {vtype}")


class GgufFile:
    """Header, metadata and tensor table of a GGUF file, its payloads as zero-copy views of a read-only map."""

    def __init__(self, path: str):
        self._f = open(path, "rb")
        self._map = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self._view = memoryview(self._map)
        c = _Cursor(self._view)
        if c.take("<I") != GGUF_MAGIC:
            raise ValueError("Invalid GGUF magic header.")
        self.version = c.take("<I")
        if self.version not in (2, 3):
            raise ValueError(f"Unsupported GGUF version: {self.version}. Supported versions: 2, 3.")
        self.tensor_count = c.take("<Q")
        self.metadata_count = c.take("<Q")
        self.metadata: dict[str, Typed] = {}
        for _ in range(self.metadata_count):
            key = c.string()
            vt = c.take("<I")
            self.metadata[key.lower()] = Typed(vt, c.value(vt))  # keys are case-insensitive in the reference
        self.alignment = self.get("general.alignment", U32, 32)
        self.tensors: list[TensorInfo] = []
        for _ in range(self.tensor_count):
            name = c.string()
            nd = c.take("<I")
            dims = [c.take("<Q") for _ in range(nd)]
            tt = c.take("<I")
            off = c.take("<Q")
            self.tensors.append(TensorInfo(name, dims, tt, off))
        a = self.alignment
        self.data_offset = (c.pos + a - 1) // a * a
        self.by_name = {t.name.lower(): t for t in self.tensors}

    def get(self, key: str, vtype: int, default):
        """GgufMetadata.GetValueOrDefault<T>: the stored value when it has the requested type, else default."""
        v = self.metadata.get(key.lower())
        if v is None or v.type != vtype:
            return default
        return v.value

    @property
    def architecture(self) -> str:
        return self.get("general.architecture", STRING, "llama")

    def tensor(self, name: str) -> TensorInfo | None:
        return self.by_name.get(name.lower())

    def tensor_bytes(self, t: TensorInfo) -> np.ndarray:
        """The payload as a read-only uint8 view of the map (no copy)."""
        start = self.data_offset + t.offset
        n = t.size_in_bytes()
        if start + n > len(self._map):
            raise ValueError(f"Tensor '{t.name}' extends beyond file boundary.")
        return np.frombuffer(self._view, dtype=np.uint8, count=n, offset=start)

    def close(self):
        """Closes the map once no tensor view of it is alive any more (until then the views keep it valid)."""
        self.by_name = {}
        try:
            self._view.release()
            self._map.close()
        except BufferError:
            pass
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def model_from_gguf(g: GgufFile) -> dict:
    """A model dictionary for `LlmEngine` (shapes + zero-copy tensor views) with LlmModel.LoadGguf's rules.
    Only Q8_0 projections and F32 norms are accepted: the device engine runs Q8_0 Llama-style models."""
    arch = g.architecture
    cfg = {
        "vocab": g.get(f"{arch}.vocab_size", U32, 32000),
        "context_length": g.get(f"{arch}.context_length", U32, 2048),
        "dim": g.get(f"{arch}.embedding_length", U32, 256),
        "layers": g.get(f"{arch}.block_count", U32, 4),
        "ffn": g.get(f"{arch}.feed_forward_length", U32, 512),
        "heads": g.get(f"{arch}.attention.head_count", U32, 4),
        "eps": g.get(f"{arch}.attention.layer_norm_rms_epsilon", F32, 1e-5),
        "rope_base": g.get(f"{arch}.rope.freq_base", F32, 10000.0),
        "bos_token": g.get("tokenizer.ggml.bos_token_id", U32, 1),
        "eos_token": g.get("tokenizer.ggml.eos_token_id", U32, 2),
    }
    cfg["kv_heads"] = g.get(f"{arch}.attention.head_count_kv", U32, cfg["heads"])
    if g.get(f"{arch}.expert_count", U32, 0) > 1 or g.get(f"{arch}.expert_shared_count", U32, 0) > 0:
        raise ValueError("mixture-of-experts GGUF models load through the MoE layer, not the dense engine")
    emb = g.tensor("token_embd.weight")
    if emb is not None and len(emb.dims) >= 2:
        cfg["dim"], cfg["vocab"] = int(emb.dims[0]), int(emb.dims[1])

    def q8(name):
        t = g.tensor(name)
        if t is None:
            raise KeyError(f"GGUF tensor '{name}' is missing")
        if t.type != T_Q8_0:
            raise ValueError(f"GGUF tensor '{name}' is not Q8_0 (type {t.type})")
        return g.tensor_bytes(t)

    def f32(name):
        t = g.tensor(name)
        if t is None:
            raise KeyError(f"GGUF tensor '{name}' is missing")
        if t.type != T_F32:
            raise ValueError(f"GGUF tensor '{name}' is not F32 (type {t.type})")
        return g.tensor_bytes(t).view(np.float32)

    m = dict(cfg)
    m["hd"] = cfg["dim"] // cfg["heads"]
    m["tok_emb"] = q8("token_embd.weight")
    m["lm_head"] = q8("output.weight") if g.tensor("output.weight") is not None else m["tok_emb"]  # tied weights
    m["final_norm"] = f32("output_norm.weight")
    L = cfg["layers"]
    per_layer = {"attn_norm": ("attn_norm", f32), "ffn_norm": ("ffn_norm", f32), "wq": ("attn_q", q8),
                 "wk": ("attn_k", q8), "wv": ("attn_v", q8), "wo": ("attn_output", q8), "wgate": ("ffn_gate", q8),
                 "wup": ("ffn_up", q8), "wdown": ("ffn_down", q8)}
    for key, (gname, fn) in per_layer.items():
        m[key] = [fn(f"blk.{l}.{gname}.weight") for l in range(L)]
    return m


def load_engine(path: str, **engine_kwargs):
    """LlmEngine over a GGUF file's Q8_0 Llama model; the map stays open for the engine's lifetime (the views
    are only read during construction, but keeping it lets callers inspect `engine.gguf`)."""
    from .engine import LlmEngine
    g = GgufFile(path)
    e = LlmEngine(model_from_gguf(g), **engine_kwargs)
    e.gguf = g
    return e


def write_gguf(path: str, metadata: list[tuple[str, int, object]], tensors: list[tuple[str, list[int], int, bytes]],
               alignment: int = 32) -> None:
    """GgufWriter.WriteTo: v3 header, typed metadata (scalars and strings), tensor infos with offsets padded to
    `alignment`, the data section aligned, every payload padded to `alignment`."""
    out = bytearray()

    def w(fmt, v):
        out.extend(struct.pack(fmt, v))

    def ws(s):
        b = s.encode("utf-8")
        w("<Q", len(b))
        out.extend(b)

    w("<I", GGUF_MAGIC)
    w("<I", 3)
    w("<Q", len(tensors))
    w("<Q", len(metadata))
    for key, vt, val in metadata:
        ws(key)
        w("<I", vt)
        if vt in _SCALAR:
            w(_SCALAR[vt], val)
        elif vt == BOOL:
            w("<B", 1 if val else 0)
        elif vt == STRING:
            ws(val)
        else:
            raise ValueError(f"Writing metadata type {vt} not supported.")
    off = 0
    for name, dims, tt, data in tensors:
        ws(name)
        w("<I", len(dims))
        for d in dims:
            w("<Q", d)
        w("<I", tt)
        w("<Q", off)
        off += (len(data) + alignment - 1) // alignment * alignment
    out.extend(b"\0" * ((-len(out)) % alignment))
    for _, _, _, data in tensors:
        out.extend(data)
        out.extend(b"\0" * ((-len(out)) % alignment))
    with open(path, "wb") as f:
        f.write(out)


def save_gguf(model: dict, path: str, arch: str = "llama", bos_token: int = 1, eos_token: int = 2) -> None:
    """LlmModel.SaveGguf for a dense Q8_0 model dictionary (the `LlmEngine` layout: Q8_0 blocks per tensor,
    per-layer tensors indexable by layer, fp32 norms)."""
    dim, vocab, L = int(model["dim"]), int(model["vocab"]), int(model["layers"])
    heads, kvh, ffn = int(model["heads"]), int(model["kv_heads"]), int(model["ffn"])
    hd = int(model.get("hd", dim // heads))
    qd, kvd = heads * hd, kvh * hd
    meta = [("general.architecture", STRING, arch), (f"{arch}.vocab_size", U32, vocab),
            (f"{arch}.context_length", U32, int(model.get("context_length", 2048))),
            (f"{arch}.embedding_length", U32, dim), (f"{arch}.block_count", U32, L),
            (f"{arch}.feed_forward_length", U32, ffn), (f"{arch}.attention.head_count", U32, heads),
            (f"{arch}.attention.head_count_kv", U32, kvh),
            (f"{arch}.attention.layer_norm_rms_epsilon", F32, float(model.get("eps", 1e-5))),
            (f"{arch}.rope.freq_base", F32, float(model.get("rope_base", 10000.0))),
            ("tokenizer.ggml.bos_token_id", U32, bos_token), ("tokenizer.ggml.eos_token_id", U32, eos_token)]

    def q8(a):
        return np.ascontiguousarray(a, dtype=np.uint8).tobytes()

    def f32(a):
        return np.ascontiguousarray(a, dtype=np.float32).tobytes()

    ts = [("token_embd.weight", [dim, vocab], T_Q8_0, q8(model["tok_emb"]))]
    for l in range(L):
        ts += [(f"blk.{l}.attn_norm.weight", [dim], T_F32, f32(model["attn_norm"][l])),
               (f"blk.{l}.attn_q.weight", [dim, qd], T_Q8_0, q8(model["wq"][l])),
               (f"blk.{l}.attn_k.weight", [dim, kvd], T_Q8_0, q8(model["wk"][l])),
               (f"blk.{l}.attn_v.weight", [dim, kvd], T_Q8_0, q8(model["wv"][l])),
               (f"blk.{l}.attn_output.weight", [qd, dim], T_Q8_0, q8(model["wo"][l])),
               (f"blk.{l}.ffn_norm.weight", [dim], T_F32, f32(model["ffn_norm"][l])),
               (f"blk.{l}.ffn_gate.weight", [dim, ffn], T_Q8_0, q8(model["wgate"][l])),
               (f"blk.{l}.ffn_up.weight", [dim, ffn], T_Q8_0, q8(model["wup"][l])),
               (f"blk.{l}.ffn_down.weight", [ffn, dim], T_Q8_0, q8(model["wdown"][l]))]
    ts += [("output_norm.weight", [dim], T_F32, f32(model["final_norm"])),
           ("output.weight", [dim, vocab], T_Q8_0, q8(model["lm_head"]))]
    write_gguf(path, meta, ts)
