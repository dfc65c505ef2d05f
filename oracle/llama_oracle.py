"""CPU restatement of one Llama decode step -- test infrastructure only.

The op order of LlamaRunner.forward (MetalLM/Backend/LlamaRunner.swift:
537-1085 per layer, 1130-1184 for the final norm and the output head),
composed from the oracle's pinned pieces (q4k_oracle.c): the bit-exact Q4_K
dequantizer in an fp64-accumulated matvec, RMSNorm (NormalizationKernels.metal:
31-79), RoPE (PositionalEmbeddingsKernels.metal:159-203) and softmax
attention in fp64.  Weights are applied in W[out][in] orientation (the
reference's MPS call reads them transposed; that is a known reference bug,
not reproduced).  Everything is fp32 (matvec sums in fp64) except the KV
cache, which is fp16 as in the reference: the reference's own fp16
activations overflow on the synthetic benchmark weights (the SiLU-gated
product exceeds 65504), so this is the fp32 composition the parity bar is
stated against.

Weights are plain numpy arrays: Q4_K tensors as uint8 block bytes
[rows * cols / 256 * 144], norms as fp32.  This module is only imported by
the tests; the product never calls it.
"""
from __future__ import annotations

from typing import Dict

import numpy as np

from . import oracle as O


def _is_q6k(W: np.ndarray, rows: int, cols: int) -> bool:
    """Q6_K block bytes (210 per 256 elements) rather than Q4_K (144)."""
    return W.dtype == np.uint8 and W.size == rows * cols // 256 * 210


def _matvec(W: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    """y = W x for a Q4_K tensor (block bytes; fp64 sums over the bit-exact
    dequantized rows), a Q6_K tensor (the bit-exact dequantization of
    DequantKernels.metal:131-172, fp64 sums) or a tensor already dequantized
    to fp32 [rows][cols] by dense() (fp32 BLAS sums)."""
    if W.dtype == np.float32:
        return W @ np.ascontiguousarray(x, dtype=np.float32)
    if _is_q6k(W, rows, cols):
        w = O.q6k_dequant_f32(W, rows * cols).reshape(rows, cols).astype(np.float64)
        return (w @ np.asarray(x, dtype=np.float64)).astype(np.float32)
    return O.q4k_matvec_f32x(W, rows, cols, x)


def layer_decode(w: Dict[str, np.ndarray], hidden: np.ndarray, kcache: np.ndarray,
                 vcache: np.ndarray, pos: int, cfg: dict) -> np.ndarray:
    """One decoder layer at position `pos`; appends K/V at row `pos` of the
    fp16 caches [max_seq][n_kv][head_dim] and returns the new fp32 hidden."""
    d, hd, nh, nkv, ffn, eps = (cfg[k] for k in ("dim", "head_dim", "n_heads", "n_kv_heads",
                                                 "ffn_dim", "rms_eps"))
    kvd = nkv * hd
    xn = O.rmsnorm_f32(hidden, w["attn_norm"], 1, d, eps)
    q = _matvec(w["wq"], d, d, xn)
    k = _matvec(w["wk"], kvd, d, xn)
    v = _matvec(w["wv"], kvd, d, xn)
    ra = O.rope_args(n_dims=hd, freq_base=cfg["rope_theta"], pos_offset=pos)
    q = O.rope_f32(ra, q, 1, nh, hd)
    k = O.rope_f32(ra, k, 1, nkv, hd)
    kcache[pos] = k.astype(np.float16).reshape(nkv, hd)
    vcache[pos] = v.astype(np.float16).reshape(nkv, hd)
    attn = O.attn_decode(q, kcache[: pos + 1], vcache[: pos + 1], nh, nkv, hd, pos + 1)
    hidden = hidden + _matvec(w["wo"], d, d, attn)
    xn2 = O.rmsnorm_f32(hidden, w["ffn_norm"], 1, d, eps)
    g = _matvec(w["w_gate"], ffn, d, xn2)
    u = _matvec(w["w_up"], ffn, d, xn2)
    return hidden + _matvec(w["w_down"], d, ffn, O.silu_mul(g, u))


def model_forward(layers, glob: Dict[str, np.ndarray], caches, token: int, pos: int,
                  cfg: dict) -> np.ndarray:
    """forward(tokenID:): embedding row, every layer, final norm, output head;
    returns fp32 logits [vocab].  caches[l] = (kcache, vcache), updated."""
    d = cfg["dim"]
    hidden = glob["tok_embd"][token * d:(token + 1) * d].astype(np.float32)
    for w, (kc, vc) in zip(layers, caches):
        hidden = layer_decode(w, hidden, kc, vc, pos, cfg)
    xn = O.rmsnorm_f32(hidden, glob["output_norm"], 1, d, cfg["rms_eps"])
    return _matvec(glob["output"], cfg["vocab"], d, xn)


def dense(w: Dict[str, np.ndarray], shapes: Dict[str, tuple]) -> Dict[str, np.ndarray]:
    """The same tensors with every Q4_K one dequantized once (bit-exact fp32,
    DequantKernels.metal:63-92) to [rows][cols]: full-size models then run
    through fp32 BLAS products instead of dequantizing per token."""
    out = dict(w)
    for name, (rows, cols) in shapes.items():
        deq = O.q6k_dequant_f32 if _is_q6k(w[name], rows, cols) else O.q4k_dequant_f32
        out[name] = deq(w[name], rows * cols).reshape(rows, cols)
    return out
