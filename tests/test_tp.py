"""Tensor-parallel host logic on CPU: gloo process groups of 2 (and 4) ranks.

- bootstrap(): rank 0's NCCL unique id reaches every rank, each joins with
  its (size, rank);
- the shard plan (metallm_b200.tp): every Q4_K tensor of a layer is covered
  exactly once by the ranks' shares, for 1/2/4/8 ranks on the Llama-3-70B
  shape;
- the sharded decoder layer (2 and 4 ranks): each rank computes its heads' attention and its
  FFN rows from its shards of the whole-model tensors, the output and down
  projections' partial sums are summed by a gloo all-reduce, and the result
  equals the oracle's whole layer (LlamaRunner.swift:537-1085) -- the
  arithmetic the GPU runner performs with NCCL.
"""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch.multiprocessing as mp

from metallm_b200.synthetic import layer_stream, llama_config, q4k_shapes
from metallm_b200.tp import Shard, bootstrap, layer_shards, output_shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int) -> None:
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))


class _FakeCtx:
    """Stands in for a Context: records the group it is asked to join."""

    def __init__(self, rank: int):
        self.rank = rank
        self.joined = None

    def tp_unique_id(self) -> bytes:
        return os.urandom(128)

    def tp_init(self, nranks: int, rank: int, uid: bytes) -> None:
        self.joined = (nranks, rank, bytes(uid))


def _bootstrap_worker(rank: int, world: int, port: int, q) -> None:
    import torch.distributed as dist
    _init(rank, world, port)
    ctx = _FakeCtx(rank)
    got = bootstrap(ctx)
    q.put((rank, got, ctx.joined))
    dist.destroy_process_group()


def _run(fn, world: int, *args) -> list:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(out, key=lambda t: t[0])


def test_bootstrap_gloo_world2():
    res = _run(_bootstrap_worker, 2)
    uids = {joined[2] for _, _, joined in res}
    assert len(uids) == 1  # one id, drawn by rank 0
    for rank, got, joined in res:
        assert got == (rank, 2)
        assert joined[:2] == (2, rank)


@pytest.mark.parametrize("size", [1, 2, 4, 8])
def test_shards_cover_each_tensor_once(size):
    cfg = llama_config(n_layers=80, dim=8192, n_heads=64, n_kv_heads=8, ffn_dim=28672)
    for name, (rows, cols) in q4k_shapes(cfg).items():
        nb = cols // 256
        seen = np.zeros((rows, nb), dtype=np.int32)
        for r in range(size):
            sh = layer_shards(cfg, Shard(r, size))[name]
            assert sh["nb"] == nb
            seen[sh["row0"]:sh["row0"] + sh["rows"], sh["kb0"]:sh["kb0"] + sh["nkb"]] += 1
        assert np.all(seen == 1), name
    covered = sum(output_shard(cfg, Shard(r, size))["rows"] for r in range(size))
    assert covered == cfg.vocab


def test_shards_reject_uneven_split():
    cfg = llama_config(n_layers=1, dim=1024, n_heads=8, n_kv_heads=2, ffn_dim=2816)
    with pytest.raises(ValueError):
        layer_shards(cfg, Shard(0, 4))  # 2 KV heads over 4 ranks


# -- the sharded layer against the oracle -------------------------------------

SEED, POS = 77, 5
CFG = dict(n_layers=1, dim=512, n_heads=4, n_kv_heads=2, ffn_dim=1024, vocab=256, max_seq=8)
# splits evenly over 4 ranks: 8 query heads, 4 KV heads, FFN 2048
CFG4 = dict(n_layers=1, dim=1024, n_heads=8, n_kv_heads=4, ffn_dim=2048, vocab=256, max_seq=8)


def _slice(blocks: np.ndarray, rows: int, nb: int, sh: dict) -> np.ndarray:
    full = blocks.reshape(rows, nb, 144)
    part = full[sh["row0"]:sh["row0"] + sh["rows"], sh["kb0"]:sh["kb0"] + sh["nkb"]]
    return np.ascontiguousarray(part).reshape(-1)


def _whole_layer(cfg):
    from oracle import oracle as O
    w = {name: O.gen_q4k(SEED, layer_stream(0, name), rows * cols // 256)
         for name, (rows, cols) in q4k_shapes(cfg).items()}
    for name in ("attn_norm", "ffn_norm"):
        w[name] = O.gen_f32(SEED, layer_stream(0, name), cfg.dim, 1.0, 0.02)
    kvd = cfg.n_kv_heads * cfg.head_dim
    caches = []
    for name in ("k_cache", "v_cache"):
        c = np.zeros((cfg.max_seq, cfg.n_kv_heads, cfg.head_dim), dtype=np.float16)
        c[:POS] = O.gen_f16(SEED, layer_stream(0, name), POS * kvd).reshape(
            POS, cfg.n_kv_heads, cfg.head_dim)
        caches.append(c)
    h = O.gen_f32(SEED, 3, cfg.dim)
    return w, caches, h


def _sharded_layer_worker(rank: int, world: int, port: int, q, cfg_kw=CFG) -> None:
    """One rank: its shard of the layer, partial sums all-reduced over gloo."""
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    _init(rank, world, port)
    cfg = llama_config(**cfg_kw)
    w, (kc, vc), h = _whole_layer(cfg)
    shard = Shard(rank, world)
    sh = layer_shards(cfg, shard)
    shapes = q4k_shapes(cfg)
    ws = {n: _slice(w[n], shapes[n][0], shapes[n][1] // 256, sh[n]) for n in shapes}
    hd, d = cfg.head_dim, cfg.dim
    nh, nkv = cfg.n_heads // world, cfg.n_kv_heads // world
    f0, f1 = shard.span(cfg.ffn_dim)
    k0, k1 = shard.span(cfg.n_kv_heads)
    eps = cfg.rms_eps
    xn = O.rmsnorm_f32(h, w["attn_norm"], 1, d, eps)
    qv = O.q4k_matvec_f32x(ws["wq"], nh * hd, d, xn)
    kv = O.q4k_matvec_f32x(ws["wk"], nkv * hd, d, xn)
    vv = O.q4k_matvec_f32x(ws["wv"], nkv * hd, d, xn)
    ra = O.rope_args(n_dims=hd, freq_base=cfg.rope.freq_base, pos_offset=POS)
    qv = O.rope_f32(ra, qv, 1, nh, hd)
    kv = O.rope_f32(ra, kv, 1, nkv, hd)
    kcl, vcl = kc[:, k0:k1].copy(), vc[:, k0:k1].copy()
    kcl[POS] = kv.astype(np.float16).reshape(nkv, hd)
    vcl[POS] = vv.astype(np.float16).reshape(nkv, hd)
    attn = O.attn_decode(qv, kcl[:POS + 1], vcl[:POS + 1], nh, nkv, hd, POS + 1)
    part = O.q4k_matvec_f32x(ws["wo"], d, nh * hd, attn)
    if rank == 0:
        part = part + h
    t = torch.from_numpy(part.astype(np.float64))
    dist.all_reduce(t)
    h1 = t.numpy()
    xn2 = O.rmsnorm_f32(h1.astype(np.float32), w["ffn_norm"], 1, d, eps)
    g = O.q4k_matvec_f32x(ws["w_gate"], f1 - f0, d, xn2)
    u = O.q4k_matvec_f32x(ws["w_up"], f1 - f0, d, xn2)
    part = O.q4k_matvec_f32x(ws["w_down"], d, f1 - f0, O.silu_mul(g, u)).astype(np.float64)
    if rank == 0:
        part = part + h1
    t = torch.from_numpy(part)
    dist.all_reduce(t)
    q.put((rank, t.numpy()))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,cfg_kw", [(2, CFG), (4, CFG4)])
def test_sharded_layer_equals_whole_layer_gloo(world, cfg_kw):
    from oracle import llama_oracle as LO
    res = _run(_sharded_layer_worker, world, cfg_kw)
    cfg = llama_config(**cfg_kw)
    w, (kc, vc), h = _whole_layer(cfg)
    cd = {"dim": cfg.dim, "head_dim": cfg.head_dim, "n_heads": cfg.n_heads,
          "n_kv_heads": cfg.n_kv_heads, "ffn_dim": cfg.ffn_dim, "rms_eps": cfg.rms_eps,
          "rope_theta": cfg.rope.freq_base, "vocab": cfg.vocab}
    want = LO.layer_decode(w, h, kc, vc, POS, cd)
    for _, got in res:
        err = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert err < 1e-5, err
