"""GGUF files: the reader and the Llama loader on this library's runner.

Replaces the reference's ``GGUFFile`` (MetalLM/Backend/Loaders/GGUF/GGUF.swift:
179-341: header, metadata key/value pairs, tensor descriptors, the data
section at the next multiple of ``general.alignment``) and the tensor side
of ``ModelLoader`` (ModelLoader.swift:104-219, 479-601; the Llama keys of
MetalLM/Models/Llama3Architecture.swift:103-138).

The loader keeps the north-star contract: the file is memory-mapped and each
Q4_K tensor's raw 144-byte blocks are uploaded unchanged into the runner's
device buffers; one in-place device repack (``mlm_q4k_repack_canonical``)
then moves every block from the GGUF element order into the order the
kernels read.  Norm weights go up as fp32; the token embedding is converted
to the runner's fp16 table on the device (F16 as is, F32 rounded, Q4_K and
Q6_K dequantized).  With tensor parallelism each rank uploads its shard
(``metallm_b200.tp``).  The linears are Q4_K, except that attn_v,
ffn_down and the output head may be Q6_K, as Q4_K_M files store them: the
runner is created with those per-tensor types (``tensor_types``) and the
Q6_K blocks go up unchanged (their GGUF order is the one the kernels read).
A file holding any other type there is rejected with the tensor's name.

``write_gguf`` writes the same format (used by the tests to build files).
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np

GGUF_MAGIC = b"GGUF"

# metadata value types (GGUF v2/v3)
VT_U8, VT_I8, VT_U16, VT_I16, VT_U32, VT_I32, VT_F32, VT_BOOL = 0, 1, 2, 3, 4, 5, 6, 7
VT_STRING, VT_ARRAY, VT_U64, VT_I64, VT_F64 = 8, 9, 10, 11, 12
_SCALAR = {VT_U8: "<B", VT_I8: "<b", VT_U16: "<H", VT_I16: "<h", VT_U32: "<I", VT_I32: "<i",
           VT_F32: "<f", VT_BOOL: "<?", VT_U64: "<Q", VT_I64: "<q", VT_F64: "<d"}

# tensor types (GGUFDataType, GGUF.swift:4-33) and (block elements, block bytes)
F32, F16, Q4_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 8, 12, 13, 14
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K",
              Q6_K: "Q6_K"}
_BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144),
          Q5_K: (256, 176), Q6_K: (256, 210)}


class GGUFError(ValueError):
    pass


@dataclass
class GGUFTensor:
    name: str
    dims: Tuple[int, ...]  # ne0 first: dims[0] is the row length (columns)
    type: int
    offset: int            # relative to the data section

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    @property
    def n_bytes(self) -> int:
        if self.type not in _BLOCK:
            raise GGUFError(f"tensor {self.name}: type {self.type} has no known block size")
        be, bb = _BLOCK[self.type]
        if self.n_elements % be:
            raise GGUFError(f"tensor {self.name}: {self.n_elements} elements, blocks of {be}")
        return self.n_elements // be * bb


class _Reader:
    def __init__(self, buf, start: int = 0):
        self.buf = buf
        self.pos = start

    def take(self, n: int) -> bytes:
        if self.pos + n > len(self.buf):
            raise GGUFError(f"truncated file: {n} bytes wanted at offset {self.pos}")
        b = self.buf[self.pos:self.pos + n]
        self.pos += n
        return bytes(b)

    def scalar(self, vt: int):
        fmt = _SCALAR[vt]
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.scalar(VT_U64)
        return self.take(n).decode("utf-8", errors="replace")

    def value(self, vt: int):
        if vt in _SCALAR:
            return self.scalar(vt)
        if vt == VT_STRING:
            return self.string()
        if vt == VT_ARRAY:
            et = self.scalar(VT_U32)
            n = self.scalar(VT_U64)
            return [self.value(et) for _ in range(n)]
        raise GGUFError(f"unknown metadata value type {vt} at offset {self.pos}")


class GGUFFile:
    """A memory-mapped GGUF file: ``metadata``, ``tensors`` (by name) and
    ``tensor_data(name)`` (a read-only uint8 view of the tensor's bytes)."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._mm = None
        try:
            self._parse()
        except BaseException:
            self.close()
            raise

    def _parse(self) -> None:
        path = self.path
        size = os.fstat(self._f.fileno()).st_size
        if size < 24:
            raise GGUFError(f"{path}: {size} bytes is too short for a GGUF header")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        r = _Reader(self._mm)
        if r.take(4) != GGUF_MAGIC:
            raise GGUFError(f"{path}: not a GGUF file (bad magic)")
        self.version = r.scalar(VT_U32)
        if self.version not in (2, 3):
            raise GGUFError(f"{path}: GGUF version {self.version} (2 and 3 are read)")
        n_tensors = r.scalar(VT_U64)
        n_kv = r.scalar(VT_U64)
        self.metadata: Dict[str, Any] = {}
        for _ in range(n_kv):
            key = r.string()
            self.metadata[key] = r.value(r.scalar(VT_U32))
        self.alignment = int(self.metadata.get("general.alignment", 32))
        self.tensors: Dict[str, GGUFTensor] = {}
        for _ in range(n_tensors):
            name = r.string()
            nd = r.scalar(VT_U32)
            dims = tuple(r.scalar(VT_U64) for _ in range(nd))
            self.tensors[name] = GGUFTensor(name, dims, r.scalar(VT_U32), r.scalar(VT_U64))
        a = self.alignment
        self.data_offset = (r.pos + a - 1) // a * a
        for t in self.tensors.values():
            if t.type in _BLOCK and self.data_offset + t.offset + t.n_bytes > size:
                raise GGUFError(f"{path}: tensor {t.name} runs past the end of the file")

    def tensor_data(self, name: str) -> np.ndarray:
        t = self.tensors.get(name)
        if t is None:
            raise GGUFError(f"{self.path}: no tensor {name}")
        start = self.data_offset + t.offset
        return np.frombuffer(self._mm, dtype=np.uint8, count=t.n_bytes, offset=start)

    def close(self) -> None:
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:  # tensor views still alive: the map goes with the last one
                pass
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def _put_value(out: List[bytes], v) -> int:
    """Append the encoding of a Python value; return its value type."""
    if isinstance(v, bool):
        out.append(struct.pack("<?", v))
        return VT_BOOL
    if isinstance(v, int):
        if 0 <= v < 2 ** 32:
            out.append(struct.pack("<I", v))
            return VT_U32
        out.append(struct.pack("<q", v))
        return VT_I64
    if isinstance(v, float):
        out.append(struct.pack("<f", v))
        return VT_F32
    if isinstance(v, str):
        b = v.encode()
        out.append(struct.pack("<Q", len(b)) + b)
        return VT_STRING
    if isinstance(v, (list, tuple)):
        body: List[bytes] = []
        et = VT_I32
        for e in v:
            et = _put_value(body, e)
        out.append(struct.pack("<IQ", et, len(v)) + b"".join(body))
        return VT_ARRAY
    raise TypeError(f"cannot encode metadata value {v!r}")


def write_gguf(path: str, metadata: Dict[str, Any],
               tensors: Sequence[Tuple[str, int, Sequence[int], np.ndarray]],
               alignment: int = 32) -> None:
    """A GGUF v3 file: metadata (ints as u32, floats as f32, strings, lists)
    and tensors given as (name, type, dims with ne0 first, raw bytes)."""
    meta = dict(metadata)
    if alignment != 32:
        meta["general.alignment"] = alignment
    head: List[bytes] = [GGUF_MAGIC, struct.pack("<IQQ", 3, len(tensors), len(meta))]
    for k, v in meta.items():
        kb = k.encode()
        body: List[bytes] = []
        vt = _put_value(body, v)
        head.append(struct.pack("<Q", len(kb)) + kb + struct.pack("<I", vt) + b"".join(body))
    offset = 0
    blobs = []
    for name, ty, dims, data in tensors:
        nb = name.encode()
        raw = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        t = GGUFTensor(name, tuple(int(d) for d in dims), ty, offset)
        if raw.size != t.n_bytes:
            raise GGUFError(f"tensor {name}: {raw.size} bytes for {t.n_bytes}")
        head.append(struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(dims)) +
                    b"".join(struct.pack("<Q", int(d)) for d in dims) +
                    struct.pack("<IQ", ty, offset))
        blobs.append((offset, raw))
        offset += (raw.size + alignment - 1) // alignment * alignment
    header = b"".join(head)
    data_start = (len(header) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(header)
        f.write(b"\0" * (data_start - len(header)))
        pos = 0
        for off, raw in blobs:
            f.write(b"\0" * (off - pos))
            f.write(raw.tobytes())
            pos = off + raw.size


# -- the Llama loader -------------------------------------------------------------

# runner tensor -> GGUF tensor name (ModelLoader.swift:561-577)
LAYER_TENSORS = {"attn_norm": "attn_norm", "wq": "attn_q", "wk": "attn_k", "wv": "attn_v",
                 "wo": "attn_output", "ffn_norm": "ffn_norm", "w_gate": "ffn_gate",
                 "w_up": "ffn_up", "w_down": "ffn_down"}


def llama_config_from_gguf(f: GGUFFile, max_seq: Optional[int] = None):
    """LlamaConfig from the metadata keys Llama3Architecture.swift:103-138 reads."""
    from . import LlamaConfig, rope_args
    arch = f.metadata.get("general.architecture", "llama")

    def key(k, default=None):
        v = f.metadata.get(f"{arch}.{k}", default)
        if v is None:
            raise GGUFError(f"{f.path}: metadata {arch}.{k} missing")
        return v

    dim = int(key("embedding_length"))
    n_heads = int(key("attention.head_count"))
    n_kv = int(key("attention.head_count_kv", n_heads))
    head_dim = dim // n_heads
    emb = f.tensors.get("token_embd.weight")
    vocab = int(key("vocab_size", emb.dims[1] if emb is not None else None))
    ctx_len = int(key("context_length", 2048))
    seq = min(ctx_len, max_seq if max_seq else 2048)
    n_rot = int(key("rope.dimension_count", head_dim))
    theta = float(key("rope.freq_base", 500000.0))
    scaling = str(key("rope.scaling.type", "none"))
    factor = float(key("rope.scaling.factor", 1.0))
    orig = int(key("rope.scaling.original_context_length", ctx_len))
    ext, fscale = 0.0, 1.0
    if scaling == "linear" and factor > 0:
        fscale = 1.0 / factor
    elif scaling == "yarn" and factor > 0:
        ext, fscale = 1.0, 1.0 / factor
    rope = rope_args(n_dims=n_rot, freq_base=theta, freq_scale=fscale, n_ctx_orig=orig,
                     ext_factor=ext, beta_fast=float(key("rope.scaling.beta_fast", 32.0)),
                     beta_slow=float(key("rope.scaling.beta_slow", 1.0)),
                     has_freq_factors="rope_freqs.weight" in f.tensors)
    return LlamaConfig(int(key("block_count")), dim, n_heads, n_kv, head_dim,
                       int(key("feed_forward_length")), vocab, seq,
                       float(key("attention.layer_norm_rms_epsilon", 1e-5)), rope)


def _check_tensor(f: GGUFFile, name: str, types: Sequence[int], rows: int, cols: int) -> GGUFTensor:
    t = f.tensors.get(name)
    if t is None:
        raise GGUFError(f"{f.path}: tensor {name} missing")
    if t.type not in types:
        want = "/".join(TYPE_NAMES.get(x, str(x)) for x in types)
        raise GGUFError(f"{f.path}: tensor {name} is {TYPE_NAMES.get(t.type, t.type)}; "
                        f"the runner takes {want} there")
    dims = tuple(t.dims) + (1,) * (2 - len(t.dims))
    if dims[:2] != (cols, rows) or any(d != 1 for d in dims[2:]):
        raise GGUFError(f"{f.path}: tensor {name} has dims {t.dims}, expected ({cols}, {rows})")
    return t


def _upload(ctx, dptr: int, data: np.ndarray) -> None:
    import ctypes
    a = np.ascontiguousarray(data)
    ctx._check(ctx.lib.mlm_upload(ctx.handle, ctypes.c_void_p(dptr), a.ctypes.data, a.nbytes),
               "mlm_upload")


BLOCK_BYTES = {Q4_K: 144, Q6_K: 210}

# linears a Q4_K_M file may store as Q6_K (the runner's typed tensors)
Q6K_OK = ("wv", "w_down")


def _block_shard(f: GGUFFile, name: str, rows: int, cols: int, sh: dict,
                 types: Sequence[int] = (Q4_K,)) -> np.ndarray:
    """The (row0, rows, kb0, nkb) part of a Q4_K (or Q6_K) tensor, [rows][nkb]
    blocks."""
    t = _check_tensor(f, name, types, rows, cols)
    full = f.tensor_data(name).reshape(rows, cols // 256, BLOCK_BYTES[t.type])
    return full[sh["row0"]:sh["row0"] + sh["rows"], sh["kb0"]:sh["kb0"] + sh["nkb"]]


def tensor_types(f: GGUFFile, n_layers: int) -> Optional[dict]:
    """The runner's per-tensor types for the file (None: all Q4_K): Q6_K
    attn_v / ffn_down / output as Q4_K_M files store them."""
    def ty(name):
        t = f.tensors.get(name)
        return t.type if t is not None else Q4_K
    out_name = "output.weight" if "output.weight" in f.tensors else "token_embd.weight"
    types = {"output": Q6_K if ty(out_name) == Q6_K else Q4_K,
             "attn_v": [Q6_K if ty(f"blk.{l}.attn_v.weight") == Q6_K else Q4_K
                        for l in range(n_layers)],
             "ffn_down": [Q6_K if ty(f"blk.{l}.ffn_down.weight") == Q6_K else Q4_K
                          for l in range(n_layers)]}
    if types["output"] == Q4_K and Q6_K not in types["attn_v"] + types["ffn_down"]:
        return None
    return types


def load_llama(ctx, path: str, max_seq: Optional[int] = None, batch: int = 1):
    """A Llama runner with the weights of a GGUF file (one rank's shard
    under tensor parallelism)."""
    from . import Llama
    from .synthetic import q4k_shapes
    from .tp import Shard, layer_shards, output_shard
    with GGUFFile(path) as f:
        cfg = llama_config_from_gguf(f, max_seq)
        m = Llama(ctx, cfg, batch, types=tensor_types(f, cfg.n_layers))
        try:
            rank, size = ctx.tp_info()
            shard = Shard(rank, max(size, 1))
            shards = layer_shards(cfg, shard)
            shapes = q4k_shapes(cfg)
            for layer in range(cfg.n_layers):
                t = m.layer_tensors(layer)
                for ours, theirs in LAYER_TENSORS.items():
                    name = f"blk.{layer}.{theirs}.weight"
                    if ours in shapes:
                        rows, cols = shapes[ours]
                        ok = (Q4_K, Q6_K) if ours in Q6K_OK else (Q4_K,)
                        blocks = _block_shard(f, name, rows, cols, shards[ours], ok)
                        _upload(ctx, t[ours], blocks)
                        if blocks.shape[-1] == 144:  # Q6_K needs no reordering
                            ctx.q4k_repack_canonical(t[ours], t[ours], blocks.size // 144)
                    else:
                        _check_tensor(f, name, (F32, F16), 1, cfg.dim)
                        _upload(ctx, t[ours], _as_f32(f, name))
            g = m.global_tensors()
            _load_embedding(ctx, f, cfg, g["tok_embd"])
            _check_tensor(f, "output_norm.weight", (F32, F16), 1, cfg.dim)
            _upload(ctx, g["output_norm"], _as_f32(f, "output_norm.weight"))
            out_name = "output.weight" if "output.weight" in f.tensors else "token_embd.weight"
            osh = output_shard(cfg, shard)
            blocks = _block_shard(f, out_name, cfg.vocab, cfg.dim,
                                  dict(row0=osh["row0"], rows=osh["rows"], kb0=0,
                                       nkb=cfg.dim // 256), (Q4_K, Q6_K))
            _upload(ctx, g["output"], blocks)
            if blocks.shape[-1] == 144:
                ctx.q4k_repack_canonical(g["output"], g["output"], blocks.size // 144)
            if cfg.rope.has_freq_factors:
                t = _check_tensor(f, "rope_freqs.weight", (F32,), 1, cfg.rope.n_dims // 2)
                _upload(ctx, g["rope_freqs"], f.tensor_data(t.name).view(np.float32))
            ctx.wait()
        except Exception:
            m.close()
            raise
    return m


def _as_f32(f: GGUFFile, name: str) -> np.ndarray:
    t = f.tensors[name]
    raw = f.tensor_data(name)
    return raw.view(np.float32) if t.type == F32 else raw.view(np.float16).astype(np.float32)


def _load_embedding(ctx, f: GGUFFile, cfg, dptr: int) -> None:
    """token_embd.weight into the runner's fp16 [vocab][dim] table."""
    name = "token_embd.weight"
    t = _check_tensor(f, name, (F16, F32, Q4_K, Q6_K), cfg.vocab, cfg.dim)
    raw = f.tensor_data(name)
    if t.type == F16:
        _upload(ctx, dptr, raw)
        return
    if t.type == F32:
        _upload(ctx, dptr, raw.view(np.float32).astype(np.float16))
        return
    import ctypes
    n = cfg.vocab * cfg.dim
    tmp = ctx.alloc(raw.size + 16)
    try:
        tmp.upload(raw)
        if t.type == Q4_K:
            ctx.q4k_repack_canonical(tmp, tmp, raw.size // 144)
            ctx.call("mlm_q4k_dequant_f16", tmp, ctypes.c_void_p(dptr), n)
        else:
            ctx.call("mlm_q6k_dequant_f16", tmp, ctypes.c_void_p(dptr), n)
        ctx.wait()
    finally:
        tmp.free()
