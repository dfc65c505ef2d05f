"""The decode runner (mlm_llama_*) against the oracle's restatement of
LlamaRunner.forward, through the C ABI.

Bar: layer output and logits within relative L2 1e-2 of the fp32/fp64
oracle composed from the bit-exact dequantizer, identical greedy argmax.
"""
from __future__ import annotations

import numpy as np
import pytest

from metallm_b200 import Llama, MLMError
from metallm_b200.synthetic import global_stream, layer_stream, llama_config, q4k_shapes
from oracle import llama_oracle as LO
from oracle import oracle as O
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-2
SEED = 2024


def cfg_dict(cfg) -> dict:
    return {"dim": cfg.dim, "head_dim": cfg.head_dim, "n_heads": cfg.n_heads,
            "n_kv_heads": cfg.n_kv_heads, "ffn_dim": cfg.ffn_dim, "rms_eps": cfg.rms_eps,
            "rope_theta": cfg.rope.freq_base, "vocab": cfg.vocab}


def oracle_layer(cfg, layer: int, types: dict | None = None) -> dict:
    """The layer's tensors as fill_llama generates them; `types` as given to
    the runner (Q6_K attn_v / ffn_down per layer)."""
    def gen(name, rows, cols):
        key = {"wv": "attn_v", "w_down": "ffn_down"}.get(name)
        q6 = types is not None and key is not None and types.get(key) is not None and \
            types[key][layer] == 14
        return (O.gen_q6k if q6 else O.gen_q4k)(SEED, layer_stream(layer, name), rows * cols // 256)
    w = {name: gen(name, rows, cols) for name, (rows, cols) in q4k_shapes(cfg).items()}
    for name in ("attn_norm", "ffn_norm"):
        w[name] = O.gen_f32(SEED, layer_stream(layer, name), cfg.dim, 1.0, 0.02)
    return w


def oracle_cache(cfg, layer: int, filled: int):
    kvd = cfg.n_kv_heads * cfg.head_dim
    caches = []
    for name in ("k_cache", "v_cache"):
        c = np.zeros((cfg.max_seq, cfg.n_kv_heads, cfg.head_dim), dtype=np.float16)
        if filled:
            c[:filled] = O.gen_f16(SEED, layer_stream(layer, name), filled * kvd).reshape(
                filled, cfg.n_kv_heads, cfg.head_dim)
        caches.append(c)
    return caches


def oracle_globals(cfg, types: dict | None = None) -> dict:
    q6 = types is not None and types.get("output") == 14
    return {"tok_embd": O.gen_f16(SEED, global_stream("tok_embd"), cfg.vocab * cfg.dim, 0.0, 0.02),
            "output_norm": O.gen_f32(SEED, global_stream("output_norm"), cfg.dim, 1.0, 0.02),
            "output": (O.gen_q6k if q6 else O.gen_q4k)(SEED, global_stream("output"),
                                                      cfg.vocab * cfg.dim // 256)}


def test_layer_decode_llama8b_shape(ctx):
    """One Llama-3-8B-shape layer, single-token decode at position 2047 over
    a 2047-token fp16 cache ~ N(0,1), fp32 input ~ N(0,1)."""
    from metallm_b200.synthetic import fill_llama
    cfg = llama_config(n_layers=1, vocab=256, max_seq=2048)
    m = Llama(ctx, cfg)
    pos = 2047
    fill_llama(m, SEED, cache_positions=pos)
    hidden = ctx.alloc(4 * cfg.dim)
    ctx.gen_f32(SEED, 7, cfg.dim, hidden)
    m.set_position(pos)
    m.forward_layer(0, hidden)
    got = hidden.download(np.float32)
    t = m.layer_tensors(0)
    kvd = cfg.n_kv_heads * cfg.head_dim
    k_row = np.empty(kvd, dtype=np.float16)
    ctx._check(ctx.lib.mlm_download(ctx.handle, k_row.ctypes.data,
                                    __import__("ctypes").c_void_p(t["k_cache"] + pos * kvd * 2),
                                    k_row.nbytes), "download")

    kc, vc = oracle_cache(cfg, 0, pos)
    want = LO.layer_decode(oracle_layer(cfg, 0), O.gen_f32(SEED, 7, cfg.dim), kc, vc, pos,
                           cfg_dict(cfg))
    assert np.all(np.isfinite(got))
    err = rel_l2(got, want)
    assert err < TOL, err
    assert rel_l2(k_row.astype(np.float32), kc[pos].reshape(-1).astype(np.float32)) < 1e-3
    m.close()


def _small_cfg():
    return llama_config(n_layers=2, dim=1024, n_heads=8, n_kv_heads=2, ffn_dim=2816,
                        vocab=4096, max_seq=64)


def test_model_forward_and_greedy(ctx):
    from metallm_b200.synthetic import fill_llama
    cfg = _small_cfg()
    m = Llama(ctx, cfg)
    fill_llama(m, SEED)
    cd = cfg_dict(cfg)
    layers = [oracle_layer(cfg, l) for l in range(cfg.n_layers)]
    glob = oracle_globals(cfg)
    caches = [oracle_cache(cfg, l, 0) for l in range(cfg.n_layers)]

    prompt = [17, 4000, 3, 999, 2048]
    logits = ctx.alloc(4 * cfg.vocab)
    for pos, tok in enumerate(prompt):
        m.forward(tok, logits)
        got = logits.download(np.float32)
        want = LO.model_forward(layers, glob, caches, tok, pos, cd)
        assert rel_l2(got, want) < TOL, (pos, rel_l2(got, want))
        assert int(np.argmax(got)) == int(np.argmax(want)), pos
    assert m.position == len(prompt)

    # greedy continuation on the device vs the oracle's argmax loop
    steps = 8
    first = int(np.argmax(want))
    out = ctx.alloc(4 * steps)
    m.decode_greedy(first, steps, out)
    got_tokens = out.download(np.int32).tolist()
    tok, pos, ref_tokens = first, len(prompt), []
    for _ in range(steps):
        lg = LO.model_forward(layers, glob, caches, tok, pos, cd)
        tok = int(np.argmax(lg))
        ref_tokens.append(tok)
        pos += 1
    assert got_tokens == ref_tokens
    assert m.position == len(prompt) + steps

    # a second greedy call replays the captured step graph
    out2 = ctx.alloc(4 * 2)
    m.decode_greedy(ref_tokens[-1], 2, out2)
    for i, g2 in enumerate(out2.download(np.int32).tolist()):
        lg = LO.model_forward(layers, glob, caches, tok, pos, cd)
        tok = int(np.argmax(lg))
        pos += 1
        assert g2 == tok, i
    m.close()


def _oracle_model(cfg, types: dict | None = None):
    layers = [oracle_layer(cfg, l, types) for l in range(cfg.n_layers)]
    return (layers, oracle_globals(cfg, types),
            [oracle_cache(cfg, l, 0) for l in range(cfg.n_layers)])


def _layer0_top2_gap(cfg, w0, glob, kcache, prompt, t: int) -> float:
    """Smallest relative gap between the two largest layer-0 attention scores
    of token t over its heads, in the oracle's fp64 arithmetic."""
    d, hd = cfg.dim, cfg.head_dim
    h = glob["tok_embd"][prompt[t] * d:(prompt[t] + 1) * d].astype(np.float32)
    xn = O.rmsnorm_f32(h, w0["attn_norm"], 1, d, cfg.rms_eps)
    q = O.q4k_matvec_f32x(w0["wq"], d, d, xn)
    q = O.rope_f32(O.rope_args(n_dims=hd, freq_base=cfg.rope.freq_base, pos_offset=t),
                   q, 1, cfg.n_heads, hd).reshape(cfg.n_heads, hd).astype(np.float64)
    k = kcache[:t + 1].astype(np.float64)
    group = cfg.n_heads // cfg.n_kv_heads
    gap = 1.0
    for hh in range(cfg.n_heads):
        s = np.sort(k[:, hh // group] @ q[hh])[::-1]
        if t > 0:
            gap = min(gap, (s[0] - s[1]) / abs(s[0]))
    return gap


@pytest.mark.parametrize("max_seq,n", [(64, 40), (1100, 1030)])
def test_prefill_vs_oracle(ctx, max_seq, n):
    """Batched prompt pass (tensor-core GEMM, bf16 activations) vs the oracle's
    token-by-token forward: last-token logits and the KV cache it leaves;
    1030 tokens cross the 1024-token chunk boundary.

    The synthetic weights give attention scores of order 1e4, so softmax is
    close to an argmax: where the two best keys of a layer-0 head are within a
    relative 2e-2 of each other, bf16 rounding of the prompt pass can pick the
    other key and that token's hidden state -- hence its layer-1 K/V row --
    differs from the fp32 oracle's.  Every layer-0 row must be within 1e-2;
    layer-1 rows carry two layers of bf16 rounding (about 8x the fp16 decode
    path's error on the same row) and must be within 2e-2 except at such
    near-tied tokens, at most 1% of them; the layer-1 cache over the other
    rows is within 1e-2.
    """
    from metallm_b200.synthetic import fill_llama
    cfg = llama_config(n_layers=2, dim=1024, n_heads=8, n_kv_heads=2, ffn_dim=2816,
                       vocab=4096, max_seq=max_seq)
    m = Llama(ctx, cfg)
    fill_llama(m, SEED)
    prompt = np.random.default_rng(n).integers(0, cfg.vocab, size=n).tolist()
    logits = ctx.alloc(4 * cfg.vocab)
    nxt = ctx.alloc(16)
    m.prefill(prompt, nxt, logits)
    got = logits.download(np.float32)
    layers, glob, caches = _oracle_model(cfg)
    for pos, tok in enumerate(prompt):
        want = LO.model_forward(layers, glob, caches, tok, pos, cfg_dict(cfg))
    assert rel_l2(got, want) < TOL, rel_l2(got, want)
    assert int(nxt.download(np.int32)[0]) == int(np.argmax(want))
    assert m.position == n
    kvd = cfg.n_kv_heads * cfg.head_dim
    for layer in range(cfg.n_layers):
        t = m.layer_tensors(layer)
        for name, idx in (("k_cache", 0), ("v_cache", 1)):
            g = np.empty(n * kvd, dtype=np.float16)
            ctx._check(ctx.lib.mlm_download(ctx.handle, g.ctypes.data,
                                            __import__("ctypes").c_void_p(t[name]), g.nbytes),
                       "dl")
            g = g.astype(np.float32).reshape(n, kvd)
            r = caches[layer][idx][:n].reshape(n, kvd).astype(np.float32)
            err = np.linalg.norm(g - r, axis=1) / np.maximum(np.linalg.norm(r, axis=1), 1e-30)
            if layer == 0:
                assert err.max() < TOL, (name, int(err.argmax()), err.max())
                continue
            bad = np.nonzero(err >= 2 * TOL)[0].tolist()
            assert len(bad) <= n // 100, (name, bad)
            for row in bad:
                gap = _layer0_top2_gap(cfg, layers[0], glob, caches[0][0], prompt, row)
                assert gap < 2e-2, (name, row, err[row], gap)
            keep = np.setdiff1d(np.arange(n), bad)
            assert rel_l2(g[keep], r[keep]) < TOL, name
    m.close()


def test_prefill_then_decode_matches_forward(ctx):
    """Prefill followed by greedy decode agrees with running forward() per token."""
    from metallm_b200.synthetic import fill_llama
    cfg = _small_cfg()
    m = Llama(ctx, cfg)
    fill_llama(m, SEED)
    prompt = [5, 6, 7, 8, 9, 10]
    la = ctx.alloc(4 * cfg.vocab)
    m.prefill(prompt, None, la)
    a = la.download(np.float32)
    m.reset()
    lb = ctx.alloc(4 * cfg.vocab)
    for tok in prompt:
        m.forward(tok, lb)
    b = lb.download(np.float32)
    assert rel_l2(a, b) < TOL
    assert int(np.argmax(a)) == int(np.argmax(b))
    m.close()


def _greedy_with_gaps(cfg, layers, glob, caches, tok, pos, steps):
    """The oracle's greedy continuation and, per step, the relative gap
    between its two largest logits."""
    out, gaps = [], []
    for _ in range(steps):
        lg = LO.model_forward(layers, glob, caches, tok, pos, cfg_dict(cfg))
        top = np.sort(lg)[::-1]
        gaps.append(float((top[0] - top[1]) / max(abs(top[0]), 1e-30)))
        tok = int(np.argmax(lg))
        out.append(tok)
        pos += 1
    return out, gaps


def test_batch_of_sequences_matches_oracle(ctx):
    """Three sequences with prompts of 5, 9 and 3 tokens, each through its own
    caches; one batched step (logits of every sequence) and a greedy batch
    continuation against the oracle's per-sequence runs.  The batched step
    feeds bf16 activations to the tensor-core GEMM, so greedy tokens must
    agree up to the first step whose oracle top-2 logits are within a
    relative 1e-3 of each other (beyond it either choice is a rounding away)."""
    from metallm_b200.synthetic import fill_llama
    cfg = _small_cfg()
    B, steps = 3, 6
    m = Llama(ctx, cfg, batch=B)
    fill_llama(m, SEED)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, cfg.vocab, size=n).tolist() for n in (5, 9, 3)]
    nxt = ctx.alloc(16)
    firsts = []
    for b, pr in enumerate(prompts):
        m.prefill(pr, nxt, None, seq=b)
        firsts.append(int(nxt.download(np.int32)[0]))
        assert m.seq_position(b) == len(pr)
    logits = ctx.alloc(4 * B * cfg.vocab)
    m.forward_batch(firsts, logits)
    got = logits.download(np.float32).reshape(B, cfg.vocab)
    want_next, oracle_state = [], []
    for b, pr in enumerate(prompts):
        layers, glob, caches = _oracle_model(cfg)
        for pos, tok in enumerate(pr):
            LO.model_forward(layers, glob, caches, tok, pos, cfg_dict(cfg))
        w = LO.model_forward(layers, glob, caches, firsts[b], len(pr), cfg_dict(cfg))
        assert rel_l2(got[b], w) < TOL, (b, rel_l2(got[b], w))
        want_next.append(int(np.argmax(w)))
        oracle_state.append((layers, glob, caches))
    assert all(m.seq_position(b) == len(pr) + 1 for b, pr in enumerate(prompts))
    out = ctx.alloc(4 * steps * B)
    m.decode_greedy_batch(want_next, steps, out)
    toks = out.download(np.int32).reshape(steps, B)
    for b, pr in enumerate(prompts):
        layers, glob, caches = oracle_state[b]
        ref, gaps = _greedy_with_gaps(cfg, layers, glob, caches, want_next[b], len(pr) + 1, steps)
        for i in range(steps):
            assert int(toks[i, b]) == ref[i], (b, i, toks[:, b].tolist(), ref, gaps)
            if gaps[i] < 1e-3:
                break
    m.close()


def test_llama_errors(ctx):
    from metallm_b200.synthetic import llama_config as lc
    with pytest.raises(MLMError) as e:
        Llama(ctx, lc(n_layers=1, dim=1000))
    assert e.value.status in (-2, -9)
    cfg = lc(n_layers=1, dim=1024, n_heads=8, n_kv_heads=2, ffn_dim=1024, vocab=512, max_seq=2)
    m = Llama(ctx, cfg)
    with pytest.raises(MLMError) as e:
        m.forward(512)
    assert e.value.status == -1
    m.forward(1)
    m.forward(2)
    with pytest.raises(MLMError) as e:
        m.forward(3)
    assert e.value.status == -8
    out = ctx.alloc(16)
    m.reset()
    with pytest.raises(MLMError) as e:
        m.decode_greedy(1, 3, out)
    assert e.value.status == -8
    m.close()


@pytest.mark.parametrize("dim,n_heads", [(1024, 8), (2048, 16)])
def test_batch_of_eight_small_groups(ctx, dim, n_heads):
    """GQA groups of 1 and 2 query heads (8 KV heads) and a batch of 8 with
    caches of 1024 positions: the fused attention's grid (8 KV heads x 8
    CTAs x 8 sequences) passes three CTAs per SM, so it stages 64-row
    phases, and the longer prompts span two phases in a CTA.  One batched
    step's logits of every sequence against the oracle's per-sequence run."""
    from metallm_b200.synthetic import fill_llama
    cfg = llama_config(n_layers=1, dim=dim, n_heads=n_heads, n_kv_heads=8, ffn_dim=1024,
                       vocab=512, max_seq=1024)
    B = 8
    m = Llama(ctx, cfg, batch=B)
    fill_llama(m, SEED)
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, cfg.vocab, size=n).tolist()
               for n in (300, 130, 70, 40, 20, 9, 3, 1)]
    nxt = ctx.alloc(16)
    firsts = []
    for b, pr in enumerate(prompts):
        m.prefill(pr, nxt, None, seq=b)
        firsts.append(int(nxt.download(np.int32)[0]))
    logits = ctx.alloc(4 * B * cfg.vocab)
    m.forward_batch(firsts, logits)
    got = logits.download(np.float32).reshape(B, cfg.vocab)
    m.close()
    for b, pr in enumerate(prompts):
        layers, glob, caches = _oracle_model(cfg)
        for pos, tok in enumerate(pr):
            LO.model_forward(layers, glob, caches, tok, pos, cfg_dict(cfg))
        w = LO.model_forward(layers, glob, caches, firsts[b], len(pr), cfg_dict(cfg))
        assert rel_l2(got[b], w) < TOL, (b, rel_l2(got[b], w))
        assert int(np.argmax(got[b])) == int(np.argmax(w)), b
