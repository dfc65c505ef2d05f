"""The runner holding a Q4_K_M file's tensor types (mlm_llama_create_typed):
a Q6_K output head and Q6_K attn_v / ffn_down in some layers, the rest
Q4_K, against the oracle over the same generated blocks (the Q6_K ones
dequantized bit-exactly as DequantKernels.metal:131-172 does,
ModelLoader.swift:274-296 picking the dequantizer by tensor type).

Decode (Q6_K GEMVs with the RMSNorm / SwiGLU stagings), the prompt pass
(Q6_K weights through the bf16 GEMM path) and a batch of sequences.
Bar: logits within relative L2 1e-2 and identical greedy tokens, as for
the all-Q4_K runner.
"""
from __future__ import annotations

import numpy as np
import pytest

from metallm_b200 import TYPE_Q4_K, TYPE_Q6_K, Context, Llama, MLMError
from metallm_b200.synthetic import fill_llama, llama_config, q4k_m_types
from oracle import llama_oracle as LO
from tests.conftest import rel_l2
from tests.test_llama_gpu import SEED, TOL, _greedy_with_gaps, _oracle_model, cfg_dict

pytestmark = pytest.mark.gpu

Q4, Q6 = TYPE_Q4_K, TYPE_Q6_K
TYPES = {"output": Q6, "attn_v": [Q6, Q4, Q6], "ffn_down": [Q6, Q6, Q4]}


def _cfg(max_seq=96):
    # the Q6_K GEMV reads 2048-column chunks: dim and FFN multiples of 2048
    return llama_config(n_layers=3, dim=2048, n_heads=16, n_kv_heads=4, ffn_dim=4096,
                        vocab=4096, max_seq=max_seq)


def test_types_reported(ctx):
    m = Llama(ctx, _cfg(), types=TYPES)
    for l in range(3):
        t = m.layer_tensors(l)
        assert t["wv_type"] == TYPES["attn_v"][l] and t["w_down_type"] == TYPES["ffn_down"][l]
    assert m.global_tensors()["output_type"] == Q6
    m.close()


def test_forward_greedy_and_prefill(ctx):
    cfg = _cfg()
    cd = cfg_dict(cfg)
    m = Llama(ctx, cfg, types=TYPES)
    fill_llama(m, SEED)
    prompt = [17, 4000, 3, 999, 2048]
    logits = ctx.alloc(4 * cfg.vocab)
    got = []
    for tok in prompt:
        m.forward(tok, logits)
        got.append(logits.download(np.float32))
    steps = 6
    first = int(np.argmax(got[-1]))
    out = ctx.alloc(4 * steps)
    m.decode_greedy(first, steps, out)
    toks = out.download(np.int32).tolist()
    # the prompt pass: 5 tokens (batched GEMV / bf16 GEMM for Q6_K) and 40
    # tokens (tensor-core GEMMs)
    long_prompt = np.random.default_rng(40).integers(0, cfg.vocab, size=40).tolist()
    pre = {}
    for pr in (prompt, long_prompt):
        m.reset()
        pl = ctx.alloc(4 * cfg.vocab)
        nxt = ctx.alloc(16)
        m.prefill(pr, nxt, pl)
        pre[len(pr)] = (pl.download(np.float32), int(nxt.download(np.int32)[0]))
    m.close()

    layers, glob, caches = _oracle_model(cfg, TYPES)
    for pos, tok in enumerate(prompt):
        want = LO.model_forward(layers, glob, caches, tok, pos, cd)
        assert rel_l2(got[pos], want) < TOL, (pos, rel_l2(got[pos], want))
        assert int(np.argmax(got[pos])) == int(np.argmax(want)), pos
    assert first == int(np.argmax(want))
    ref, gaps = _greedy_with_gaps(cfg, layers, glob, caches, first, len(prompt), steps)
    assert toks == ref, (toks, ref, gaps)
    assert rel_l2(pre[5][0], got[-1]) < TOL and pre[5][1] == first
    layers, glob, caches = _oracle_model(cfg, TYPES)
    for pos, tok in enumerate(long_prompt):
        want = LO.model_forward(layers, glob, caches, tok, pos, cd)
    assert rel_l2(pre[40][0], want) < TOL, rel_l2(pre[40][0], want)
    assert pre[40][1] == int(np.argmax(want))


def test_batch_of_sequences(ctx):
    """Three sequences: prompt passes, one batched step and a greedy batch
    continuation (Q6_K rows one GEMV per row, the Q6_K head too) against
    the oracle's per-sequence runs.  The batched step feeds the Q4_K linears
    bf16 activations; the synthetic Q6_K weights (int8 scales times q - 32)
    are several times larger than the Q4_K ones, so that rounding moves this
    model's logits by about 2e-3 relative (the prompt pass against the
    single-token step measures 2.1e-3): greedy tokens must agree up to the
    first step whose oracle top-2 logits are within a relative 1e-2 (at and
    beyond it either choice is a rounding away)."""
    cfg = _cfg()
    B, steps = 3, 4
    m = Llama(ctx, cfg, batch=B, types=TYPES)
    fill_llama(m, SEED)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, cfg.vocab, size=n).tolist() for n in (5, 9, 3)]
    nxt = ctx.alloc(16)
    firsts = []
    for b, pr in enumerate(prompts):
        m.prefill(pr, nxt, None, seq=b)
        firsts.append(int(nxt.download(np.int32)[0]))
    logits = ctx.alloc(4 * B * cfg.vocab)
    m.forward_batch(firsts, logits)
    got = logits.download(np.float32).reshape(B, cfg.vocab)
    want_next = []
    states = []
    for b, pr in enumerate(prompts):
        layers, glob, caches = _oracle_model(cfg, TYPES)
        for pos, tok in enumerate(pr):
            LO.model_forward(layers, glob, caches, tok, pos, cfg_dict(cfg))
        w = LO.model_forward(layers, glob, caches, firsts[b], len(pr), cfg_dict(cfg))
        assert rel_l2(got[b], w) < TOL, (b, rel_l2(got[b], w))
        want_next.append(int(np.argmax(w)))
        states.append((layers, glob, caches))
    out = ctx.alloc(4 * steps * B)
    m.decode_greedy_batch(want_next, steps, out)
    toks = out.download(np.int32).reshape(steps, B)
    for b, pr in enumerate(prompts):
        layers, glob, caches = states[b]
        ref, gaps = _greedy_with_gaps(cfg, layers, glob, caches, want_next[b], len(pr) + 1, steps)
        for i in range(steps):
            if gaps[i] < 1e-2:  # a near-tie: either token is a rounding away
                break
            assert int(toks[i, b]) == ref[i], (b, i, toks[:, b].tolist(), ref, gaps)
    m.close()


def test_q4_k_m_recipe_and_limits(ctx):
    t = q4k_m_types(32)
    assert t["output"] == Q6 and len(t["attn_v"]) == 32
    assert t["attn_v"][0] == Q6 and t["attn_v"][31] == Q6 and Q4 in t["attn_v"]
    # Q6_K tensors need 2048-column chunks per rank
    bad = llama_config(n_layers=1, dim=1024, n_heads=8, n_kv_heads=2, ffn_dim=2048, vocab=512,
                       max_seq=8)
    with pytest.raises(MLMError) as e:
        Llama(ctx, bad, types={"output": Q6})
    assert e.value.status == -9
    with pytest.raises(MLMError) as e:
        Llama(ctx, _cfg(), types={"output": 13})
    assert e.value.status == -9


def test_group_of_one():
    """The sharded code path (partial sums, all-reduce, argmax keys) with
    Q6_K tensors, on a one-rank group."""
    cfg = _cfg()
    with Context(0) as c:
        c.tp_init(1, 0, c.tp_unique_id())
        m = Llama(c, cfg, types=TYPES)
        fill_llama(m, SEED)
        logits = c.alloc(4 * cfg.vocab)
        prompt = [9, 8, 7]
        got = []
        for tok in prompt:
            m.forward(tok, logits)
            got.append(logits.download(np.float32))
        m.close()
    layers, glob, caches = _oracle_model(cfg, TYPES)
    for pos, tok in enumerate(prompt):
        want = LO.model_forward(layers, glob, caches, tok, pos, cfg_dict(cfg))
        assert rel_l2(got[pos], want) < TOL, (pos, rel_l2(got[pos], want))
        assert int(np.argmax(got[pos])) == int(np.argmax(want))
