"""GGUF reader / writer and the Llama config mapping on CPU.

- write_gguf -> GGUFFile round trip: metadata of every kind the loader
  reads (u32, f32, strings, bools, arrays), tensors of F32 / F16 / Q4_K /
  Q6_K at the default and a larger alignment, byte for byte;
- llama_config_from_gguf reads the keys of Llama3Architecture.swift:103-138
  (RoPE theta default 500000, YaRN and linear scaling);
- malformed files (bad magic, a tensor past the end of the file) and a
  linear of an unsupported type are rejected with the reason.
"""
from __future__ import annotations

import numpy as np
import pytest

from metallm_b200 import gguf as G
from oracle import oracle as O


def _meta(**over):
    m = {"general.architecture": "llama", "llama.block_count": 2,
         "llama.embedding_length": 1024, "llama.feed_forward_length": 3072,
         "llama.attention.head_count": 8, "llama.attention.head_count_kv": 2,
         "llama.attention.layer_norm_rms_epsilon": 1e-5, "llama.context_length": 8192,
         "llama.vocab_size": 4096, "tokenizer.ggml.tokens": ["a", "b", "<s>"],
         "tokenizer.ggml.token_type": [1, 1, 3], "general.quantized": True}
    m.update(over)
    return m


@pytest.mark.parametrize("alignment", [32, 64])
def test_write_read_round_trip(tmp_path, alignment):
    q4 = O.gen_q4k(1, 2, 16)
    q6 = O.gen_q6k(1, 3, 3)
    f32 = O.gen_f32(1, 4, 100)
    f16 = O.gen_f16(1, 5, 77)
    path = str(tmp_path / "m.gguf")
    tensors = [("a.q4", G.Q4_K, (1024, 4), q4), ("b.q6", G.Q6_K, (256, 3), q6),
               ("c.f32", G.F32, (100,), f32), ("d.f16", G.F16, (7, 11), f16)]
    G.write_gguf(path, _meta(), tensors, alignment=alignment)
    with G.GGUFFile(path) as f:
        assert f.version == 3 and f.alignment == alignment
        assert f.metadata["llama.block_count"] == 2
        assert abs(f.metadata["llama.attention.layer_norm_rms_epsilon"] - 1e-5) < 1e-12
        assert f.metadata["tokenizer.ggml.tokens"] == ["a", "b", "<s>"]
        assert f.metadata["tokenizer.ggml.token_type"] == [1, 1, 3]
        assert f.metadata["general.quantized"] is True
        assert f.data_offset % alignment == 0
        for name, ty, dims, data in tensors:
            t = f.tensors[name]
            assert (t.type, t.dims) == (ty, dims)
            assert t.offset % alignment == 0
            assert np.array_equal(f.tensor_data(name), data.view(np.uint8).reshape(-1))


def test_llama_config_keys(tmp_path):
    path = str(tmp_path / "c.gguf")
    G.write_gguf(path, _meta(**{"llama.rope.freq_base": 10000.0}), [])
    with G.GGUFFile(path) as f:
        c = G.llama_config_from_gguf(f, max_seq=512)
    assert (c.n_layers, c.dim, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn_dim, c.vocab,
            c.max_seq) == (2, 1024, 8, 2, 128, 3072, 4096, 512)
    assert c.rope.freq_base == 10000.0 and c.rope.ext_factor == 0.0 and not c.rope.has_freq_factors
    G.write_gguf(path, _meta(**{"llama.rope.scaling.type": "yarn",
                                "llama.rope.scaling.factor": 4.0,
                                "llama.rope.scaling.original_context_length": 8192}), [])
    with G.GGUFFile(path) as f:
        c = G.llama_config_from_gguf(f)
    assert c.rope.freq_base == 500000.0  # the reference's default
    assert c.rope.ext_factor == 1.0 and c.rope.freq_scale == 0.25 and c.rope.n_ctx_orig == 8192
    assert c.max_seq == 2048


def test_malformed_files_are_rejected(tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + b"\0" * 60)
    with pytest.raises(G.GGUFError, match="magic"):
        G.GGUFFile(str(bad))
    path = str(tmp_path / "t.gguf")
    G.write_gguf(path, _meta(), [("w", G.Q4_K, (256, 8), O.gen_q4k(2, 2, 8))])
    raw = open(path, "rb").read()
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(raw[:-100])
    with pytest.raises(G.GGUFError, match="past the end"):
        G.GGUFFile(str(trunc))
    v1 = bytearray(raw)
    v1[4:8] = (1).to_bytes(4, "little")
    (tmp_path / "v1.gguf").write_bytes(bytes(v1))
    with pytest.raises(G.GGUFError, match="version"):
        G.GGUFFile(str(tmp_path / "v1.gguf"))


def test_linear_of_another_type_is_named(tmp_path):
    path = str(tmp_path / "q6.gguf")
    G.write_gguf(path, _meta(), [("blk.0.attn_v.weight", G.Q6_K, (1024, 256),
                                  O.gen_q6k(3, 1, 1024))])
    with G.GGUFFile(path) as f:
        with pytest.raises(G.GGUFError, match="blk.0.attn_v.weight is Q6_K"):
            G._check_tensor(f, "blk.0.attn_v.weight", (G.Q4_K,), 256, 1024)


@pytest.mark.parametrize("size", [1, 2, 4])
def test_loader_shards_tile_each_tensor(tmp_path, size):
    """The blocks each rank's loader uploads (its tensor-parallel shard of a
    GGUF tensor) put together give the whole tensor exactly once."""
    from metallm_b200.synthetic import llama_config, q4k_shapes
    from metallm_b200.tp import Shard, layer_shards, output_shard
    cfg = llama_config(n_layers=1, dim=1024, n_heads=8, n_kv_heads=4, ffn_dim=2048, vocab=512)
    shapes = q4k_shapes(cfg)
    tensors = [(f"blk.0.{G.LAYER_TENSORS[n]}.weight", G.Q4_K, (c, r),
                O.gen_q4k(9, i, r * c // 256)) for i, (n, (r, c)) in enumerate(shapes.items())]
    tensors.append(("output.weight", G.Q4_K, (cfg.dim, cfg.vocab),
                    O.gen_q4k(9, 99, cfg.vocab * cfg.dim // 256)))
    path = str(tmp_path / "s.gguf")
    G.write_gguf(path, _meta(), tensors)
    with G.GGUFFile(path) as f:
        for name, (rows, cols) in shapes.items():
            full = f.tensor_data(f"blk.0.{G.LAYER_TENSORS[name]}.weight").reshape(rows, cols // 256, 144)
            seen = np.zeros(full.shape[:2], dtype=np.int32)
            for r in range(size):
                sh = layer_shards(cfg, Shard(r, size))[name]
                part = G._block_shard(f, f"blk.0.{G.LAYER_TENSORS[name]}.weight", rows, cols, sh)
                sl = (slice(sh["row0"], sh["row0"] + sh["rows"]), slice(sh["kb0"], sh["kb0"] + sh["nkb"]))
                assert np.array_equal(part, full[sl])
                seen[sl] += 1
            assert np.all(seen == 1), name
        out = f.tensor_data("output.weight").reshape(cfg.vocab, cfg.dim // 256, 144)
        parts = []
        for r in range(size):
            osh = output_shard(cfg, Shard(r, size))
            parts.append(G._block_shard(f, "output.weight", cfg.vocab, cfg.dim,
                                      dict(row0=osh["row0"], rows=osh["rows"], kb0=0,
                                           nkb=cfg.dim // 256)))
        assert np.array_equal(np.concatenate(parts), out)


def test_failed_parse_closes_the_file(tmp_path):
    """A file rejected while parsing leaves no open handle behind."""
    import gc
    import os
    bad = tmp_path / "short.gguf"
    bad.write_bytes(b"GGUF" + (3).to_bytes(4, "little") + b"\xff" * 40)  # counts past the end
    fd_dir = f"/proc/{os.getpid()}/fd"
    before = len(os.listdir(fd_dir)) if os.path.isdir(fd_dir) else None
    for _ in range(20):
        with pytest.raises(G.GGUFError):
            G.GGUFFile(str(bad))
    gc.collect()
    if before is not None:
        assert len(os.listdir(fd_dir)) <= before + 1


def test_tensor_types_of_a_q4_k_m_file(tmp_path):
    """Per-tensor types as the runner takes them: Q6_K attn_v / ffn_down /
    output found by name; an all-Q4_K file gives None."""
    path = str(tmp_path / "types.gguf")
    G.write_gguf(path, _meta(), [
        ("blk.0.attn_v.weight", G.Q6_K, (1024, 256), O.gen_q6k(3, 1, 1024)),
        ("blk.0.ffn_down.weight", G.Q4_K, (1024, 256), O.gen_q4k(3, 2, 1024)),
        ("output.weight", G.Q6_K, (1024, 256), O.gen_q6k(3, 3, 1024))])
    with G.GGUFFile(path) as f:
        t = G.tensor_types(f, 2)
    assert t == {"output": G.Q6_K, "attn_v": [G.Q6_K, G.Q4_K], "ffn_down": [G.Q4_K, G.Q4_K]}
    path2 = str(tmp_path / "plain.gguf")
    G.write_gguf(path2, _meta(), [("output.weight", G.Q4_K, (1024, 256), O.gen_q4k(3, 3, 1024))])
    with G.GGUFFile(path2) as f:
        assert G.tensor_types(f, 2) is None
