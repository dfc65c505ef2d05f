"""The GGUF loader on the GPU: a Llama-shaped file in the GGUF element order
loads into a runner that computes exactly what the directly filled runner
computes.

The file is written from the oracle's generators (the streams fill_llama
uses), with every Q4_K tensor converted to the GGUF element order; the
loader uploads the raw blocks and repacks them on the device, so the two
runners hold identical bytes: their logits and greedy tokens must be equal
bit for bit (on one GPU, and on two ranks under tensor parallelism when two
GPUs are present).  A Q4_K token embedding is dequantized at load to the
reference kernel's fp16 values.
"""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest

from metallm_b200 import Context, Llama
from metallm_b200 import gguf as G
from metallm_b200.synthetic import (fill_llama, global_stream, layer_stream, llama_config,
                                    q4k_shapes)
from oracle import oracle as O

pytestmark = pytest.mark.gpu

SEED = 5
PROMPT = [17, 4000, 3, 999, 2048]


def _cfg():
    return llama_config(n_layers=2, dim=1024, n_heads=8, n_kv_heads=2, ffn_dim=3072,
                        vocab=4096, max_seq=64)


def interleaved_to_gguf(blocks: np.ndarray) -> np.ndarray:
    """Q4_K blocks from the kernels' element order to the GGUF order."""
    b = blocks.reshape(-1, 144).copy()
    qs = b[:, 16:]
    nib = np.stack([qs & 0xF, qs >> 4], axis=-1).reshape(-1, 4, 2, 32)  # [blk][j][half][l]
    b[:, 16:] = (nib[:, :, 0, :] | (nib[:, :, 1, :] << 4)).reshape(-1, 128)
    return b.reshape(-1)


def write_model(path: str, cfg, embd_q4k: bool = False, types: dict | None = None) -> None:
    """A Llama GGUF file from the fill_llama streams; `types` (as given to the
    runner) stores attn_v / ffn_down / output as Q6_K where it says so."""
    meta = {"general.architecture": "llama", "llama.block_count": cfg.n_layers,
            "llama.embedding_length": cfg.dim, "llama.feed_forward_length": cfg.ffn_dim,
            "llama.attention.head_count": cfg.n_heads,
            "llama.attention.head_count_kv": cfg.n_kv_heads,
            "llama.attention.layer_norm_rms_epsilon": float(cfg.rms_eps),
            "llama.rope.freq_base": float(cfg.rope.freq_base),
            "llama.context_length": cfg.max_seq, "llama.vocab_size": cfg.vocab}
    tensors = []
    names = dict(G.LAYER_TENSORS)
    for l in range(cfg.n_layers):
        for ours, (rows, cols) in q4k_shapes(cfg).items():
            key = {"wv": "attn_v", "w_down": "ffn_down"}.get(ours)
            if types and key and types[key][l] == G.Q6_K:
                w = O.gen_q6k(SEED, layer_stream(l, ours), rows * cols // 256)
                tensors.append((f"blk.{l}.{names[ours]}.weight", G.Q6_K, (cols, rows), w))
                continue
            w = O.gen_q4k(SEED, layer_stream(l, ours), rows * cols // 256)
            tensors.append((f"blk.{l}.{names[ours]}.weight", G.Q4_K, (cols, rows),
                            interleaved_to_gguf(w)))
        for ours in ("attn_norm", "ffn_norm"):
            tensors.append((f"blk.{l}.{ours}.weight", G.F32, (cfg.dim,),
                            O.gen_f32(SEED, layer_stream(l, ours), cfg.dim, 1.0, 0.02)))
    if embd_q4k:
        e = O.gen_q4k(SEED, 991, cfg.vocab * cfg.dim // 256)
        tensors.append(("token_embd.weight", G.Q4_K, (cfg.dim, cfg.vocab), e))
    else:
        tensors.append(("token_embd.weight", G.F16, (cfg.dim, cfg.vocab),
                        O.gen_f16(SEED, global_stream("tok_embd"), cfg.vocab * cfg.dim, 0.0,
                                  0.02)))
    tensors.append(("output_norm.weight", G.F32, (cfg.dim,),
                    O.gen_f32(SEED, global_stream("output_norm"), cfg.dim, 1.0, 0.02)))
    if types and types["output"] == G.Q6_K:
        out = O.gen_q6k(SEED, global_stream("output"), cfg.vocab * cfg.dim // 256)
        tensors.append(("output.weight", G.Q6_K, (cfg.dim, cfg.vocab), out))
    else:
        out = O.gen_q4k(SEED, global_stream("output"), cfg.vocab * cfg.dim // 256)
        tensors.append(("output.weight", G.Q4_K, (cfg.dim, cfg.vocab), interleaved_to_gguf(out)))
    G.write_gguf(path, meta, tensors)


def _run(ctx, m, cfg):
    logits = ctx.alloc(4 * cfg.vocab)
    lgs = []
    for tok in PROMPT:
        m.forward(tok, logits)
        lgs.append(logits.download(np.float32))
    out = ctx.alloc(4 * 4)
    m.decode_greedy(int(np.argmax(lgs[-1])), 4, out)
    return np.stack(lgs), out.download(np.int32)


def test_loaded_runner_equals_filled_runner(ctx, tmp_path):
    cfg = _cfg()
    path = str(tmp_path / "llama.gguf")
    write_model(path, cfg)
    m = G.load_llama(ctx, path, max_seq=64)
    assert (m.cfg.n_layers, m.cfg.dim, m.cfg.vocab) == (2, 1024, 4096)
    got = _run(ctx, m, cfg)
    m.close()
    ref = Llama(ctx, cfg)
    fill_llama(ref, SEED)
    want = _run(ctx, ref, cfg)
    ref.close()
    assert np.array_equal(got[0], want[0])
    assert np.array_equal(got[1], want[1])


def test_q4_k_m_file_loads_with_its_types(ctx, tmp_path):
    """A Q4_K_M-style file (Q6_K output head, Q6_K attn_v / ffn_down in some
    layers): the loader creates the runner with those types, uploads the
    Q6_K blocks unchanged and repacks only the Q4_K ones; the loaded runner
    equals the directly filled typed runner bit for bit."""
    cfg = llama_config(n_layers=3, dim=2048, n_heads=16, n_kv_heads=4, ffn_dim=4096,
                       vocab=4096, max_seq=64)
    types = {"output": G.Q6_K, "attn_v": [G.Q6_K, G.Q4_K, G.Q6_K],
             "ffn_down": [G.Q6_K, G.Q6_K, G.Q4_K]}
    path = str(tmp_path / "q4km.gguf")
    write_model(path, cfg, types=types)
    with G.GGUFFile(path) as f:
        assert G.tensor_types(f, cfg.n_layers) == types
    m = G.load_llama(ctx, path, max_seq=64)
    assert m.layer_tensors(0)["wv_type"] == G.Q6_K and m.global_tensors()["output_type"] == G.Q6_K
    got = _run(ctx, m, cfg)
    m.close()
    ref = Llama(ctx, cfg, types=types)
    fill_llama(ref, SEED)
    want = _run(ctx, ref, cfg)
    ref.close()
    assert np.array_equal(got[0], want[0])
    assert np.array_equal(got[1], want[1])


def test_q4k_embedding_dequantized_at_load(ctx, tmp_path):
    cfg = _cfg()
    path = str(tmp_path / "llama_q4e.gguf")
    write_model(path, cfg, embd_q4k=True)
    m = G.load_llama(ctx, path, max_seq=64)
    import ctypes
    host = np.empty(cfg.vocab * cfg.dim, dtype=np.float16)
    ctx._check(ctx.lib.mlm_download(ctx.handle, host.ctypes.data,
                                    ctypes.c_void_p(m.global_tensors()["tok_embd"]), host.nbytes),
               "mlm_download")
    m.close()
    with G.GGUFFile(path) as f:
        raw = np.array(f.tensor_data("token_embd.weight"))
    want = O.q4k_dequant_f16(O.q4k_canonical_to_interleaved(raw), cfg.vocab * cfg.dim)
    assert np.array_equal(host.view(np.uint16), want.view(np.uint16))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_worker(rank: int, world: int, port: int, path: str, q) -> None:
    import torch.distributed as dist

    from metallm_b200.tp import bootstrap
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        with Context(rank) as c:
            bootstrap(c)
            m = G.load_llama(c, path, max_seq=64)
            got = _run(c, m, _cfg())
            m.close()
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_two_ranks_load_their_shards(ctx, tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = _cfg()
    path = str(tmp_path / "llama_tp.gguf")
    write_model(path, cfg)
    ref = Llama(ctx, cfg)
    fill_llama(ref, SEED)
    want = _run(ctx, ref, cfg)
    ref.close()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_rank_worker, args=(r, 2, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in (0, 1):
        assert np.array_equal(res[r][1], want[1])  # greedy tokens
        rel = np.linalg.norm(res[r][0] - want[0]) / np.linalg.norm(want[0])
        assert rel < 1e-2, rel  # the sums are split over the ranks
