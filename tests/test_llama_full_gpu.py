"""The runner at the full sizes of the Llama-3-8B and -70B shapes against the
oracle, through the C ABI.

- Llama-3-8B shape: all 32 layers, vocab 128256, Q4_K output head.  An
  8-token prompt token by token (mlm_llama_forward), 4 greedy steps in the
  captured decode graph, and the same prompt through the batched prompt pass
  (mlm_llama_prefill).
- Llama-3-70B shape: one layer (hidden 8192, 64 query / 8 KV heads, FFN
  28672) with a small head, alone and under a tensor-parallel group of one
  rank (the sharded code path: partial sums and all-reduces).

The oracle is the reference's op order (LlamaRunner.swift:537-1085 per
layer, 1130-1184 for the norm and head) over the bit-exact dequantized
weights (oracle.llama_oracle.dense: each Q4_K tensor dequantized once, fp32
products).  Bar: logits within relative L2 1e-2, identical argmax, and the
same greedy tokens.
"""
from __future__ import annotations

import numpy as np
import pytest

from metallm_b200 import Context, Llama
from metallm_b200.synthetic import fill_llama, llama_config, q4k_shapes
from oracle import llama_oracle as LO
from tests.conftest import rel_l2
from tests.test_llama_gpu import SEED, TOL, cfg_dict, oracle_cache, oracle_globals, oracle_layer

pytestmark = pytest.mark.gpu


def _dense_model(cfg):
    shapes = q4k_shapes(cfg)
    layers = [LO.dense(oracle_layer(cfg, l), shapes) for l in range(cfg.n_layers)]
    glob = LO.dense(oracle_globals(cfg), {"output": (cfg.vocab, cfg.dim)})
    caches = [oracle_cache(cfg, l, 0) for l in range(cfg.n_layers)]
    return layers, glob, caches


def _run_and_check(ctx, cfg, prompt, steps, prefill=True):
    m = Llama(ctx, cfg)
    fill_llama(m, SEED)
    logits = ctx.alloc(4 * cfg.vocab)
    got = []
    for tok in prompt:
        m.forward(tok, logits)
        got.append(logits.download(np.float32))
    first = int(np.argmax(got[-1]))
    out = ctx.alloc(4 * steps)
    m.decode_greedy(first, steps, out)
    got_tokens = out.download(np.int32).tolist()
    pre = None
    if prefill:
        m.reset()
        pl = ctx.alloc(4 * cfg.vocab)
        nxt = ctx.alloc(16)
        m.prefill(prompt, nxt, pl)
        pre = (pl.download(np.float32), int(nxt.download(np.int32)[0]))
    m.close()

    layers, glob, caches = _dense_model(cfg)
    cd = cfg_dict(cfg)
    for pos, tok in enumerate(prompt):
        want = LO.model_forward(layers, glob, caches, tok, pos, cd)
        err = rel_l2(got[pos], want)
        assert err < TOL, (pos, err)
        assert int(np.argmax(got[pos])) == int(np.argmax(want)), pos
    last = want
    tok, pos, ref_tokens = first, len(prompt), []
    for _ in range(steps):
        lg = LO.model_forward(layers, glob, caches, tok, pos, cd)
        tok = int(np.argmax(lg))
        ref_tokens.append(tok)
        pos += 1
    assert got_tokens == ref_tokens
    if pre is not None:
        # the prompt pass runs bf16 activations into the tensor-core GEMM
        err = rel_l2(pre[0], last)
        assert err < TOL, err
        assert pre[1] == int(np.argmax(last))


def test_llama8b_all_layers_full_vocab(ctx):
    cfg = llama_config(n_layers=32, vocab=128256, max_seq=64)
    prompt = [128000, 17, 4000, 3, 99999, 2048, 12345, 77]
    _run_and_check(ctx, cfg, prompt, steps=4)


def _cfg70_layer():
    return llama_config(n_layers=1, dim=8192, n_heads=64, n_kv_heads=8, ffn_dim=28672,
                        vocab=2048, max_seq=64)


PROMPT70 = [5, 1999, 42, 1024, 7]


def test_llama70b_layer(ctx):
    _run_and_check(ctx, _cfg70_layer(), PROMPT70, steps=3)


def test_llama70b_layer_group_of_one():
    with Context(0) as c:
        c.tp_init(1, 0, c.tp_unique_id())
        assert c.tp_info() == (0, 1)
        _run_and_check(c, _cfg70_layer(), PROMPT70, steps=3)
