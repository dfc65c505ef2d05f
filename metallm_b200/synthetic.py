"""Seeded synthetic Llama weights and caches for the decode runner.

No checkpoint is used anywhere: a model of a named shape is filled on the
device by the counter-based generators of the C ABI (mlm_gen_q4k / _f16 /
_f32), which the CPU oracle reproduces bit for bit.  Every tensor has its
own generator stream, given here, so a CPU restatement can rebuild any
tensor on its own.

Distributions (the benchmark configurations): Q4_K blocks with d, dmin =
fp16(|N(0,1)| * 0.01), 6-bit scales/mins uniform, nibbles uniform; RMSNorm
weights 1 + N(0, 0.02) fp32; token embedding N(0, 0.02) fp16; KV-cache
entries N(0, 1) fp16.
"""
from __future__ import annotations

from typing import Dict

from ._lib import LlamaConfig, rope_args

LAYER_TENSORS = ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "attn_norm", "ffn_norm",
                 "k_cache", "v_cache")
GLOBAL_TENSORS = ("tok_embd", "output_norm", "output")


def layer_stream(layer: int, name: str) -> int:
    return 1000 + 100 * layer + LAYER_TENSORS.index(name)


def global_stream(name: str) -> int:
    return 500 + GLOBAL_TENSORS.index(name)


def llama_config(n_layers: int = 32, dim: int = 4096, n_heads: int = 32, n_kv_heads: int = 8,
                 ffn_dim: int = 14336, vocab: int = 128256, max_seq: int = 2048,
                 rms_eps: float = 1e-5, rope_theta: float = 500000.0) -> LlamaConfig:
    """Llama-3-8B shape by default (head_dim 128, RoPE theta 500000, YaRN off)."""
    return LlamaConfig(n_layers, dim, n_heads, n_kv_heads, 128, ffn_dim, vocab, max_seq, rms_eps,
                       rope_args(n_dims=128, freq_base=rope_theta))


def q4k_shapes(cfg: LlamaConfig) -> Dict[str, tuple]:
    """(rows, cols) of each Q4_K tensor of a layer (GGUF: cols = ne0)."""
    kvd = cfg.n_kv_heads * cfg.head_dim
    return {"wq": (cfg.dim, cfg.dim), "wk": (kvd, cfg.dim), "wv": (kvd, cfg.dim),
            "wo": (cfg.dim, cfg.dim), "w_gate": (cfg.ffn_dim, cfg.dim),
            "w_up": (cfg.ffn_dim, cfg.dim), "w_down": (cfg.dim, cfg.ffn_dim)}


def _fill_q4k(ctx, seed: int, stream: int, sh: dict, out, q6: bool = False) -> None:
    """The (row0, rows, kb0, nkb) part of generated tensor `stream` (Q4_K, or
    Q6_K when q6)."""
    if sh["kb0"] == 0 and sh["nkb"] == sh["nb"]:
        gen = ctx.gen_q6k if q6 else ctx.gen_q4k
        gen(seed, stream, sh["rows"] * sh["nb"], out, first_block=sh["row0"] * sh["nb"])
    else:
        sub = ctx.gen_q6k_sub if q6 else ctx.gen_q4k_sub
        sub(seed, stream, sh["nb"], sh["row0"], sh["rows"], sh["kb0"], sh["nkb"], out)


# tensors of a layer whose type the runner reports (a Q4_K_M file's Q6_K ones)
TYPED = {"wv": "wv_type", "w_down": "w_down_type"}


def q4k_m_types(n_layers: int) -> dict:
    """The per-tensor types llama.cpp's Q4_K_M recipe gives a Llama model:
    Q6_K output head, Q6_K attn_v and ffn_down in the first and last eighth
    of the layers and in every third layer between, Q4_K elsewhere."""
    def q6(l):
        return l < n_layers // 8 or l >= 7 * n_layers // 8 or (l - n_layers // 8) % 3 == 2
    t = [14 if q6(l) else 12 for l in range(n_layers)]
    return {"output": 14, "attn_v": t, "ffn_down": list(t)}


def fill_llama(llama, seed: int, cache_positions: int = 0, layers=None) -> None:
    """Fill the runner's weights (and the first `cache_positions` rows of
    every layer's KV cache) on the device.  Under tensor parallelism each
    rank fills exactly its shard of the same whole model (metallm_b200.tp),
    so every group size computes the same network."""
    from .tp import Shard, layer_shards, output_shard
    ctx, cfg = llama.ctx, llama.cfg
    rank, size = ctx.tp_info()
    shard = Shard(rank, max(size, 1))
    if size and cache_positions:
        raise ValueError("prefilled caches are not generated under tensor parallelism")
    kvd = cfg.n_kv_heads * cfg.head_dim
    shards = layer_shards(cfg, shard)
    for layer in (range(cfg.n_layers) if layers is None else layers):
        t = llama.layer_tensors(layer)
        for name in q4k_shapes(cfg):
            q6 = name in TYPED and t[TYPED[name]] == 14
            _fill_q4k(ctx, seed, layer_stream(layer, name), shards[name], t[name], q6)
        for name in ("attn_norm", "ffn_norm"):
            ctx.gen_f32(seed, layer_stream(layer, name), cfg.dim, t[name], 1.0, 0.02)
        if cache_positions:
            for name in ("k_cache", "v_cache"):
                ctx.gen_f16(seed, layer_stream(layer, name), cache_positions * kvd, t[name])
    g = llama.global_tensors()
    ctx.gen_f16(seed, global_stream("tok_embd"), cfg.vocab * cfg.dim, g["tok_embd"], 0.0, 0.02)
    ctx.gen_f32(seed, global_stream("output_norm"), cfg.dim, g["output_norm"], 1.0, 0.02)
    _fill_q4k(ctx, seed, global_stream("output"), output_shard(cfg, shard), g["output"],
              g["output_type"] == 14)
