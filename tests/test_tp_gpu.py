"""Tensor-parallel runner on the GPU, through the C ABI.

- mlm_gen_q4k_sub reproduces the slice of the whole generated tensor;
- a one-rank NCCL group runs the sharded code path (partial sums, NCCL
  all-reduce and the argmax-key all-gather inside the captured greedy step)
  on one GPU: logits and greedy tokens against the oracle as for the
  single-GPU runner (relative L2 1e-2, identical argmax);
- with two or more GPUs, two ranks (one process each, NCCL over NVLink)
  hold half of the model each and must give the same logits and tokens.
"""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from metallm_b200 import Context, Llama
from metallm_b200.synthetic import fill_llama, llama_config
from oracle import llama_oracle as LO
from oracle import oracle as O
from tests.conftest import rel_l2
from tests.test_llama_gpu import SEED, TOL, _oracle_model, cfg_dict

pytestmark = pytest.mark.gpu

PROMPT = [17, 4000, 3, 999, 2048]
STEPS = 6
BATCH_PROMPTS = [[11, 22, 33, 44], [3000, 7]]
BATCH_NEXT = [5, 4095]


def _tp_cfg():
    # every split even for 2 ranks: 8 heads, 2 KV heads, FFN 3072, vocab 4096
    return llama_config(n_layers=2, dim=1024, n_heads=8, n_kv_heads=2, ffn_dim=3072,
                        vocab=4096, max_seq=64)


def _oracle_run(cfg):
    """Per-token logits of PROMPT, then STEPS greedy tokens, from the oracle."""
    layers, glob, caches = _oracle_model(cfg)
    cd = cfg_dict(cfg)
    lgs = [LO.model_forward(layers, glob, caches, t, p, cd) for p, t in enumerate(PROMPT)]
    tok, pos, toks = int(np.argmax(lgs[-1])), len(PROMPT), []
    first = tok
    for _ in range(STEPS):
        lg = LO.model_forward(layers, glob, caches, tok, pos, cd)
        tok = int(np.argmax(lg))
        toks.append(tok)
        pos += 1
    return lgs, first, toks


def _device_run(ctx, cfg):
    m = Llama(ctx, cfg)
    fill_llama(m, SEED)
    logits = ctx.alloc(4 * cfg.vocab)
    lgs = []
    for tok in PROMPT:
        m.forward(tok, logits)
        lgs.append(logits.download(np.float32))
    first = int(np.argmax(lgs[-1]))
    out = ctx.alloc(4 * STEPS)
    m.decode_greedy(first, STEPS, out)
    toks = out.download(np.int32).tolist()
    # the batched prompt pass on the same group: last logits
    m.reset()
    pl = ctx.alloc(4 * cfg.vocab)
    nxt = ctx.alloc(16)
    m.prefill(PROMPT, nxt, pl)
    pre = (pl.download(np.float32), int(nxt.download(np.int32)[0]))
    m.close()
    # a batch of two sequences: both prompts, then one batched step
    mb = Llama(ctx, cfg, batch=2)
    fill_llama(mb, SEED)
    for b, pr in enumerate(BATCH_PROMPTS):
        mb.prefill(pr, nxt, None, seq=b)
    bl = ctx.alloc(4 * 2 * cfg.vocab)
    mb.forward_batch(BATCH_NEXT, bl)
    btoks = ctx.alloc(4 * 2 * 3)
    mb.decode_greedy_batch(BATCH_NEXT, 3, btoks)
    batch = (bl.download(np.float32).reshape(2, cfg.vocab), btoks.download(np.int32).reshape(3, 2))
    mb.close()
    return lgs, first, toks, pre, batch


def _check(cfg, got):
    lgs, first, toks, (pre_lg, pre_next), (blg, _) = got
    for b, pr in enumerate(BATCH_PROMPTS):  # the batched step, per sequence
        layers, glob, caches = _oracle_model(cfg)
        for pos, tok in enumerate(pr):
            LO.model_forward(layers, glob, caches, tok, pos, cfg_dict(cfg))
        w = LO.model_forward(layers, glob, caches, BATCH_NEXT[b], len(pr), cfg_dict(cfg))
        assert rel_l2(blg[b], w) < TOL, (b, rel_l2(blg[b], w))
        assert int(np.argmax(blg[b])) == int(np.argmax(w)), b
    want_lgs, want_first, want_toks = _oracle_run(cfg)
    for p, (g, w) in enumerate(zip(lgs, want_lgs)):
        assert rel_l2(g, w) < TOL, (p, rel_l2(g, w))
        assert int(np.argmax(g)) == int(np.argmax(w)), p
    assert first == want_first
    assert toks == want_toks
    assert rel_l2(pre_lg, want_lgs[-1]) < TOL
    assert pre_next == int(np.argmax(want_lgs[-1]))


def test_gen_q4k_sub_matches_slice(ctx):
    rows, nb = 96, 12
    full = O.gen_q4k(5, 9, rows * nb).reshape(rows, nb, 144)
    out = ctx.alloc(40 * 5 * 144)
    ctx.gen_q4k_sub(5, 9, nb, 17, 40, 3, 5, out)
    got = out.download(np.uint8).reshape(40, 5, 144)
    assert np.array_equal(got, full[17:57, 3:8])


def test_group_of_one_runs_sharded_path():
    cfg = _tp_cfg()
    with Context(0) as c:
        c.tp_init(1, 0, c.tp_unique_id())
        assert c.tp_info() == (0, 1)
        got = _device_run(c, cfg)
    _check(cfg, got)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_worker(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist

    from metallm_b200.tp import bootstrap
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        with Context(rank) as c:
            bootstrap(c)
            got = _device_run(c, _tp_cfg())
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_two_ranks_match_oracle():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    cfg = _tp_cfg()
    for rank in (0, 1):
        _check(cfg, res[rank])
    # both ranks drew the same greedy tokens for the batch
    assert np.array_equal(res[0][4][1], res[1][4][1])
