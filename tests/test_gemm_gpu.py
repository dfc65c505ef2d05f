"""Prefill Q4_K GEMM on the tensor cores (mlm_q4k_gemm), through the C ABI.

Bar: relative L2 <= 2e-3 against a float64 product of the same bf16
operands (the exact fp32 dequantization rounded to bf16, x in bf16).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 2e-3


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even), as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = u + 0x7FFF + ((u >> 16) & 1)
    return (u >> 16).astype(np.uint16)


def bf16_value(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _run(ctx, rows, cols, tokens, seed=5):
    nb = rows * cols // 256
    blocks = O.gen_q4k(seed, 1, nb)
    xb = bf16_bits(O.gen_f32(seed, 2, tokens * cols))
    y = ctx.alloc(4 * rows * tokens)
    ctx.call("mlm_q4k_gemm", ctx.to_device(blocks), rows, cols, ctx.to_device(xb), tokens, y, None)
    got = y.download(np.float32, rows * tokens).reshape(tokens, rows)
    w = bf16_value(bf16_bits(O.q4k_dequant_f32(blocks, rows * cols))).reshape(rows, cols)
    x = bf16_value(xb).reshape(tokens, cols)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    return got, ref


@pytest.mark.parametrize("rows,cols,tokens", [(128, 256, 512), (256, 1024, 512), (200, 768, 100),
                                              (4096, 4096, 512), (1000, 2048, 1300),
                                              (6144, 4096, 64),
                                              # one token tile: the MMA shrinks to 16 .. 256
                                              (4096, 4096, 1), (2048, 1024, 8), (1000, 2048, 17),
                                              (512, 512, 250)])
def test_gemm_shapes(ctx, rows, cols, tokens):
    got, ref = _run(ctx, rows, cols, tokens)
    assert np.all(np.isfinite(got))
    err = rel_l2(got, ref)
    assert err < TOL, (rows, cols, tokens, err)


@pytest.mark.parametrize("rows,cols,tokens", [(4096, 4096, 512), (1000, 2048, 1300),
                                              (8192, 1024, 8)])
def test_gemm_residual_in_place(ctx, rows, cols, tokens):
    """y = x W^T + y (the residual stream updated in place), split and unsplit."""
    nb = rows * cols // 256
    blocks = O.gen_q4k(6, 1, nb)
    xb = bf16_bits(O.gen_f32(6, 2, tokens * cols))
    r = O.gen_f32(6, 3, tokens * rows, 0.0, 100.0)
    y = ctx.to_device(r)
    ctx.call("mlm_q4k_gemm", ctx.to_device(blocks), rows, cols, ctx.to_device(xb), tokens, y, y)
    got = y.download(np.float32, rows * tokens).reshape(tokens, rows)
    w = bf16_value(bf16_bits(O.q4k_dequant_f32(blocks, rows * cols))).reshape(rows, cols)
    ref = bf16_value(xb).reshape(tokens, cols).astype(np.float64) @ w.astype(np.float64).T
    ref += r.reshape(tokens, rows)
    assert rel_l2(got, ref) < TOL


def gemm_schedule(sm_count: int, rows: int, cols: int, tokens: int) -> dict:
    """The launch plan of mlm_q4k_gemm (q4k_gemm.cu, gemm_launch): output
    tiles of 256 rows x 256 tokens, one persistent CTA per SM with at least
    16 K stages each, whole-tile waves first and one to two waves' worth of
    tiles left to stream-K."""
    tiles = -(-rows // 256) * -(-tokens // 256)
    ks = cols // 256 * 8
    ctas = min(sm_count, -(-tiles * ks // 16))
    return {"tiles": tiles, "ctas": ctas, "dp_waves": max(0, tiles // ctas - 1)}


def _sample_rows(rows: int, n: int, seed: int) -> np.ndarray:
    return np.sort(np.random.default_rng(seed).choice(rows, size=min(rows, n), replace=False))


@pytest.mark.parametrize("rows,cols,tokens,sample,in_place", [
    # 320 tiles: one whole-tile wave, then stream-K
    (20480, 256, 1024, 0, False),
    (20480, 256, 1024, 0, True),
    # the 8B gate/up on a 2048-token prompt (896 tiles, 5 whole-tile waves)
    (28672, 4096, 2048, 384, False),
    (28672, 4096, 2048, 384, True),
    # a 16384-token product (1024 tiles)
    (4096, 4096, 16384, 256, False),
    # the 70B gate/up on a 1024-token prompt chunk (896 tiles)
    (57344, 8192, 1024, 256, False),
])
def test_gemm_whole_tile_waves(ctx, rows, cols, tokens, sample, in_place):
    """Launches large enough that CTAs take whole output tiles before the
    stream-K split (dp_waves >= 1).  Large products are checked on a seeded
    sample of weight rows (every token of each sampled row)."""
    sm = ctx.lib.mlm_device_sm_count(ctx.handle)
    plan = gemm_schedule(sm, rows, cols, tokens)
    assert plan["dp_waves"] >= 1, plan
    nb = rows * cols // 256
    seed = 40 + rows % 7
    blocks = O.gen_q4k(seed, 1, nb)
    xb = bf16_bits(O.gen_f32(seed, 2, tokens * cols))
    if in_place:
        r = O.gen_f32(seed, 3, tokens * rows, 0.0, 100.0)
        y = ctx.to_device(r)
        res = y
    else:
        r = None
        y = ctx.alloc(4 * rows * tokens)
        res = None
    ctx.call("mlm_q4k_gemm", ctx.to_device(blocks), rows, cols, ctx.to_device(xb), tokens, y, res)
    got = y.download(np.float32, rows * tokens).reshape(tokens, rows)
    bpr = cols // 256 * 144  # bytes of one weight row
    sel = np.arange(rows) if sample == 0 else _sample_rows(rows, sample, seed)
    wb = blocks.reshape(rows, bpr)[sel].reshape(-1)
    w = bf16_value(bf16_bits(O.q4k_dequant_f32(wb, len(sel) * cols))).reshape(len(sel), cols)
    x = bf16_value(xb).reshape(tokens, cols)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    if r is not None:
        ref += r.reshape(tokens, rows)[:, sel]
    g = got[:, sel]
    assert np.all(np.isfinite(g))
    err = rel_l2(g, ref)
    assert err < TOL, (rows, cols, tokens, plan, err)


def test_gemm_bad_args(ctx):
    from metallm_b200 import MLMError
    buf = ctx.alloc(1 << 16)
    with pytest.raises(MLMError) as e:
        ctx.call("mlm_q4k_gemm", buf, 128, 300, buf, 16, buf, None)
    assert e.value.status == -2
    with pytest.raises(MLMError) as e:
        ctx.call("mlm_q4k_gemm", buf.ptr + 8, 128, 256, buf, 16, buf, None)
    assert e.value.status == -3


# -- the decode linears of a batch of 1..8 tokens (mlm_q4k_gemv_batch) ---------
# Bar: relative L2 <= 1e-5 against a float64 product of the exact fp32
# dequantized weights and the bf16 tokens (the weights are not rounded here;
# x goes to fp16 with a power-of-two scale per sub-block, which is exact for
# bf16 values in range).

GEMV_TOL = 1e-5


@pytest.mark.parametrize("rows,cols,tokens,scale", [(4096, 4096, 8, 1.0), (1000, 2048, 3, 1.0),
                                                    (6144, 4096, 5, 1.0), (300, 512, 1, 1.0),
                                                    (4096, 14336, 8, 1.0),
                                                    # a 70B rank's shares at 4 GPUs: narrower
                                                    # K chunks (2 block columns), and a last
                                                    # chunk of 4 of 8 columns
                                                    (8192, 2048, 8, 1.0), (2560, 8192, 8, 1.0),
                                                    (8192, 7168, 8, 1.0),
                                                    # beyond the fp16 range: the scales hold it
                                                    (2048, 1024, 4, 3.0e5)])
def test_gemv_batch(ctx, rows, cols, tokens, scale):
    nb = rows * cols // 256
    blocks = O.gen_q4k(9, 1, nb)
    xb = bf16_bits(O.gen_f32(9, 2, tokens * cols) * np.float32(scale))
    r = O.gen_f32(9, 3, tokens * rows, 0.0, 10.0)
    y = ctx.to_device(r)
    ctx.call("mlm_q4k_gemv_batch", ctx.to_device(blocks), rows, cols, ctx.to_device(xb), tokens,
             y, y)
    got = y.download(np.float32, rows * tokens).reshape(tokens, rows)
    w = O.q4k_dequant_f32(blocks, rows * cols).reshape(rows, cols).astype(np.float64)
    ref = bf16_value(xb).reshape(tokens, cols).astype(np.float64) @ w.T
    ref += r.reshape(tokens, rows)
    assert rel_l2(got, ref) < GEMV_TOL, rel_l2(got, ref)
    # and without a residual: y is written from zero
    y2 = ctx.alloc(4 * rows * tokens)
    ctx.call("mlm_q4k_gemv_batch", ctx.to_device(blocks), rows, cols, ctx.to_device(xb), tokens,
             y2, None)
    got2 = y2.download(np.float32, rows * tokens).reshape(tokens, rows)
    assert rel_l2(got2, ref - r.reshape(tokens, rows)) < GEMV_TOL


def test_gemv_batch_bad_args(ctx):
    from metallm_b200 import MLMError
    buf = ctx.alloc(1 << 16)
    with pytest.raises(MLMError):
        ctx.call("mlm_q4k_gemv_batch", buf, 128, 256, buf, 9, buf, None)  # > 8 tokens
    with pytest.raises(MLMError):
        ctx.call("mlm_q4k_gemv_batch", buf, 128, 300, buf, 2, buf, None)  # cols % 256
