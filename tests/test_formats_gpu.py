"""Q6_K and the GGUF Q4_K element order on the GPU, through the C ABI.

- mlm_gen_q6k writes the oracle generator's bytes;
- mlm_q6k_dequant_f32 is bit-exact against the oracle (itself bit-exact
  against the reference's kernel_dequantize_q6_K_f32); the fp16 / bf16
  forms are the rounding of those values;
- mlm_q6k_gemv: relative L2 <= 1e-5 against the oracle's fp64-accumulated
  dequant dot product, with and without the residual, ragged row counts;
- mlm_q4k_repack_canonical equals the oracle repack byte for byte (out of
  place and in place, partial and whole 128-block groups), and a GEMV on
  repacked GGUF-order weights matches the GGUF-order dequant dot product.
"""
from __future__ import annotations

import numpy as np
import pytest

from metallm_b200 import MLMError
from oracle import oracle as O
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-5


@pytest.mark.parametrize("nblocks,first", [(1, 0), (37, 5), (4096, 100)])
def test_gen_q6k_matches_oracle(ctx, nblocks, first):
    out = ctx.alloc(nblocks * 210 + 16)
    ctx.gen_q6k(21, 3, nblocks, out, first_block=first)
    got = out.download(np.uint8, nblocks * 210)
    assert np.array_equal(got, O.gen_q6k(21, 3, nblocks, first_block=first))


@pytest.mark.parametrize("nblocks", [1, 9, 65536])
def test_q6k_dequant_bit_exact(ctx, nblocks):
    n = nblocks * 256
    blocks = O.gen_q6k(8, 1, nblocks)
    db = ctx.to_device(blocks)
    want = O.q6k_dequant_f32(blocks, n)
    out = ctx.alloc(4 * n)
    ctx.q6k_dequant_f32(db, out, n)
    assert np.array_equal(out.download(np.uint32, n), want.view(np.uint32))
    h = ctx.alloc(2 * n)
    ctx.q6k_dequant_f16(db, h, n)
    assert np.array_equal(h.download(np.float16, n), want.astype(np.float16))
    ctx.q6k_dequant_bf16(db, h, n)
    got_bf = h.download(np.uint16, n).astype(np.uint32) << 16
    want_bf = want.view(np.uint32)
    # round to nearest even on the top 16 bits
    rnd = (want_bf + 0x7FFF + ((want_bf >> 16) & 1)) & 0xFFFF0000
    assert np.array_equal(got_bf, rnd)


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1024, 4096), (4096, 14336), (7, 2048),
                                       (333, 8192)])
def test_q6k_gemv(ctx, rows, cols):
    nb = rows * cols // 256
    W = O.gen_q6k(31, 2, nb)
    x = O.gen_f16(31, 5, cols)
    want = O.q6k_matvec(W, rows, cols, x)
    dW, dx = ctx.to_device(W), ctx.to_device(x)
    y = ctx.alloc(4 * rows)
    ctx.q6k_gemv(dW, rows, cols, dx, y)
    got = y.download(np.float32, rows)
    assert rel_l2(got, want) < GEMV_TOL
    res = O.gen_f32(31, 6, rows)
    ctx.q6k_gemv(dW, rows, cols, dx, y, ctx.to_device(res))
    assert rel_l2(y.download(np.float32, rows), want + res) < GEMV_TOL


def test_q6k_gemv_rejects_bad_shapes(ctx):
    W = ctx.alloc(210 * 64)
    x = ctx.alloc(2 * 4096)
    y = ctx.alloc(4 * 64)
    with pytest.raises(MLMError):
        ctx.q6k_gemv(W, 16, 1024, x, y)  # cols not a multiple of 2048
    with pytest.raises(MLMError):
        ctx.q6k_gemv(W, 1, 65536, x, y)  # above the 32768-column limit


@pytest.mark.parametrize("nblocks", [1, 127, 128, 129, 100_000])
def test_q4k_repack_matches_oracle(ctx, nblocks):
    b = O.gen_q4k(41, 9, nblocks)
    want = O.q4k_canonical_to_interleaved(b)
    src = ctx.to_device(b)
    dst = ctx.alloc(b.size)
    ctx.q4k_repack_canonical(src, dst, nblocks)
    assert np.array_equal(dst.download(np.uint8, b.size), want)
    ctx.q4k_repack_canonical(src, src, nblocks)  # in place
    assert np.array_equal(src.download(np.uint8, b.size), want)


def test_q4k_repack_rejects_partial_overlap(ctx):
    buf = ctx.alloc(144 * 64)
    with pytest.raises(MLMError):  # dst starts 16 blocks into the 32-block source
        ctx.call("mlm_q4k_repack_canonical", buf, buf.ptr + 144 * 16, 32)


def test_gemv_on_repacked_gguf_weights(ctx):
    rows, cols = 512, 4096
    nb = rows * cols // 256
    b = O.gen_q4k(43, 2, nb)  # read as GGUF-order blocks
    x = O.gen_f16(43, 3, cols)
    dense = O.q4k_dequant_canonical_f32(b, rows * cols).reshape(rows, cols).astype(np.float64)
    want = dense @ x.astype(np.float64)
    W = ctx.to_device(b)
    ctx.q4k_repack_canonical(W, W, nb)
    y = ctx.alloc(4 * rows)
    ctx.q4k_gemv(W, rows, cols, ctx.to_device(x), y)
    assert rel_l2(y.download(np.float32, rows), want) < GEMV_TOL


# -- the Q6_K linears of Q4_K_M files inside the model ----------------------------

def _q6_dense(W, rows, cols):
    return O.q6k_dequant_f32(W, rows * cols).reshape(rows, cols).astype(np.float64)


def test_q6k_gemv_scaled_x(ctx):
    """x = x_f16 * x_scale[k/32] (the down projection's input format)."""
    rows, cols = 1000, 14336
    W = O.gen_q6k(41, 1, rows * cols // 256)
    x16 = O.gen_f16(41, 2, cols)
    scale = (2.0 ** (np.arange(cols // 32) % 9)).astype(np.float32)
    r = O.gen_f32(41, 3, rows)
    y = ctx.alloc(4 * rows)
    ctx.call("mlm_q6k_gemv_xs", ctx.to_device(W), rows, cols, ctx.to_device(x16),
             ctx.to_device(scale), y, ctx.to_device(r))
    xtrue = x16.astype(np.float64) * np.repeat(scale, 32)
    ref = _q6_dense(W, rows, cols) @ xtrue + r
    assert rel_l2(y.download(np.float32), ref) < GEMV_TOL


def test_q6k_gemv_rmsnorm_input(ctx):
    """x = fp16(RMSNorm(hidden)) formed inside the Q6_K GEMV (attn_v, output)."""
    import ctypes
    rows, cols = 1024, 4096
    W = O.gen_q6k(42, 1, rows * cols // 256)
    h = O.gen_f32(42, 2, cols, 0.0, 3.0)
    w = O.gen_f32(42, 3, cols, 1.0, 0.02)
    y = ctx.alloc(4 * rows)
    ctx.call("mlm_q6k_gemv_rmsnorm", ctx.to_device(W), rows, cols, ctx.to_device(h),
             ctx.to_device(w), ctypes.c_float(1e-5), y, None)
    xn = O.rmsnorm_f32(h, w, 1, cols, 1e-5).astype(np.float16)
    ref = O.q6k_matvec(W, rows, cols, xn)
    assert rel_l2(y.download(np.float32), ref) < GEMV_TOL


def test_q6k_gemv_swiglu_input(ctx):
    """x = silu(gate) * up formed inside the Q6_K GEMV (ffn_down), with the
    residual; large values go to fp16 with a power-of-two scale."""
    rows, cols = 4096, 14336
    W = O.gen_q6k(43, 1, rows * cols // 256)
    g = O.gen_f32(43, 2, cols, 0.0, 200.0)
    u = O.gen_f32(43, 3, cols, 0.0, 200.0)
    r = O.gen_f32(43, 4, rows)
    y = ctx.alloc(4 * rows)
    ctx.call("mlm_q6k_gemv_swiglu", ctx.to_device(W), rows, cols, ctx.to_device(g),
             ctx.to_device(u), y, ctx.to_device(r))
    ref = _q6_dense(W, rows, cols) @ O.silu_mul(g, u).astype(np.float64) + r
    got = y.download(np.float32)
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) < 1e-3  # x rounded to fp16 (2^-11 per element)


def _bf16_round(a):
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16
    return u.view(np.float32)


@pytest.mark.parametrize("rows,cols,tokens,in_place", [
    (1024, 4096, 512, False), (4096, 14336, 64, True), (1000, 2048, 17, False),
    (300, 4096, 1, True),
    # 320 output tiles: whole-tile waves before the stream-K split
    (20480, 2048, 1024, False)])
def test_q6k_gemm(ctx, rows, cols, tokens, in_place):
    """The prompt linears on a Q6_K weight: dequantized to bf16 into the
    scratch, then the tensor-core GEMM on it; relative L2 <= 2e-3 against the
    fp64 product of the same bf16 operands."""
    W = O.gen_q6k(44, 1, rows * cols // 256)
    xf = O.gen_f32(44, 2, tokens * cols)
    xb = (_bf16_round(xf).view(np.uint32) >> 16).astype(np.uint16)
    r = O.gen_f32(44, 3, tokens * rows, 0.0, 10.0)
    scratch = ctx.alloc(2 * rows * cols)
    if in_place:
        y = ctx.to_device(r)
        res = y
    else:
        y = ctx.alloc(4 * rows * tokens)
        res = None
    ctx.call("mlm_q6k_gemm", ctx.to_device(W), rows, cols, ctx.to_device(xb), tokens, y, res,
             scratch)
    got = y.download(np.float32, rows * tokens).reshape(tokens, rows)
    w = _bf16_round(O.q6k_dequant_f32(W, rows * cols)).reshape(rows, cols).astype(np.float64)
    ref = _bf16_round(xf).reshape(tokens, cols).astype(np.float64) @ w.T
    if in_place:
        ref += r.reshape(tokens, rows)
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) < 2e-3
