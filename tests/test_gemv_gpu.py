"""GPU parity of the fused Q4_K x fp16 decode GEMV, through the C ABI.

Bar: relative L2 <= 1e-5 against the oracle's fp64-accumulated product of the
bit-exact fp32 dequantization (the reference runs the product in MPS on the
dequantized weights).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _run(ctx, rows, cols, seed=11, residual=False):
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(seed, 1, nb, W)
    x = ctx.alloc(2 * cols)
    ctx.gen_f16(seed, 2, cols, x)
    y = ctx.alloc(4 * rows)
    r = None
    if residual:
        r = ctx.alloc(4 * rows)
        ctx.gen_f32(seed, 3, rows, r)
    ctx.q4k_gemv(W, rows, cols, x, y, r)
    got = y.download(np.float32)
    ref = O.q4k_matvec(O.gen_q4k(seed, 1, nb), rows, cols, O.gen_f16(seed, 2, cols), acc64=True)
    if residual:
        ref = ref + O.gen_f32(seed, 3, rows)
    return got, ref


def test_gemv_golden(ctx, golden):
    rows, cols = (int(v) for v in golden["mv_shape"])
    W = ctx.to_device(golden["mv_W"])
    x = ctx.to_device(golden["mv_x"])
    y = ctx.alloc(4 * rows)
    ctx.q4k_gemv(W, rows, cols, x, y)
    assert rel_l2(y.download(np.float32), golden["mv_y"]) < TOL


@pytest.mark.parametrize("rows,cols", [(256, 256), (16, 256), (1, 512), (100, 512),
                                       (33, 4096), (4096, 4096), (1024, 14336), (3000, 768)])
def test_gemv_shapes(ctx, rows, cols):
    got, ref = _run(ctx, rows, cols)
    assert rel_l2(got, ref) < TOL, (rows, cols)


def test_gemv_llama8b_ffn_up(ctx):
    got, ref = _run(ctx, 14336, 4096)
    assert rel_l2(got, ref) < TOL


def test_gemv_llama8b_ffn_down(ctx):
    got, ref = _run(ctx, 4096, 14336)
    assert rel_l2(got, ref) < TOL


def test_gemv_residual(ctx):
    got, ref = _run(ctx, 777, 2048, residual=True)
    assert rel_l2(got, ref) < TOL


def test_gemv_deterministic_and_repeatable(ctx):
    """Split-K partials are summed in a fixed order; counters reset per launch."""
    rows, cols = 4096, 14336
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(5, 1, nb, W)
    x = ctx.alloc(2 * cols)
    ctx.gen_f16(5, 2, cols, x)
    y = ctx.alloc(4 * rows)
    outs = []
    for _ in range(3):
        ctx.q4k_gemv(W, rows, cols, x, y)
        outs.append(y.download(np.uint32))
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])


def test_gemv_linearity(ctx):
    """W(x1 + x2) = W x1 + W x2 within tolerance (x1 + x2 exact in fp16)."""
    rows, cols = 2048, 4096
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(9, 1, nb, W)
    x1 = (O.gen_f16(9, 2, cols).astype(np.float32) * 0.5).astype(np.float16)
    x2 = (O.gen_f16(9, 3, cols).astype(np.float32) * 0.25).astype(np.float16)
    xs = (x1.astype(np.float32) + x2.astype(np.float32)).astype(np.float16)
    ys = []
    for xv in (x1, x2, xs):
        y = ctx.alloc(4 * rows)
        ctx.q4k_gemv(W, rows, cols, ctx.to_device(xv), y)
        ys.append(y.download(np.float32).astype(np.float64))
    # x1 + x2 rounds in fp16 where needed; compare against the oracle on xs instead
    ref = O.q4k_matvec(O.gen_q4k(9, 1, nb), rows, cols, xs)
    assert rel_l2(ys[2], ref) < TOL
    assert rel_l2(ys[0] + ys[1], ys[2]) < 1e-3


def test_gemv_rejects_bad_shapes(ctx):
    from metallm_b200 import MLMError
    W = ctx.alloc(144 * 4)
    x = ctx.alloc(2 * 512)
    y = ctx.alloc(4 * 4)
    with pytest.raises(MLMError) as e:
        ctx.q4k_gemv(W, 2, 300, x, y)  # cols not a multiple of 256
    assert e.value.status == -2
    with pytest.raises(MLMError) as e:
        ctx.q4k_gemv(W.ptr + 8, 2, 256, x, y)
    assert e.value.status == -3


def test_gemv_graph_replay_matches_eager(ctx):
    """A captured sequence of GEMVs (with programmatic dependent launch) replays exactly."""
    rows, cols = 14336, 4096
    nb = rows * cols // 256
    Ws = []
    for c in range(3):
        W = ctx.alloc(nb * 144)
        ctx.gen_q4k(50 + c, 1, nb, W)
        Ws.append(W)
    x = ctx.alloc(2 * cols)
    ctx.gen_f16(50, 2, cols, x)
    ys = [ctx.alloc(4 * rows) for _ in range(3)]
    for c in range(3):
        ctx.q4k_gemv(Ws[c], rows, cols, x, ys[c])
    eager = [y.download(np.uint32) for y in ys]
    for y in ys:
        ctx.call("mlm_memset", y, 0, y.nbytes)
    ctx.graph_begin()
    for c in range(3):
        ctx.q4k_gemv(Ws[c], rows, cols, x, ys[c])
    g = ctx.graph_end()
    for _ in range(2):
        g.launch()
    ctx.wait()
    g.destroy()
    for c in range(3):
        assert np.array_equal(ys[c].download(np.uint32), eager[c])
    ref = O.q4k_matvec(O.gen_q4k(52, 1, nb), rows, cols, O.gen_f16(50, 2, cols))
    assert rel_l2(ys[2].download(np.float32), ref) < TOL


def test_gemv_scaled_x(ctx):
    """x = x_f16 * x_scale[k/32]: the down projection's input format."""
    rows, cols = 1000, 14336
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(21, 1, nb, W)
    x16 = O.gen_f16(21, 2, cols)
    scale = (2.0 ** (np.arange(cols // 32) % 9)).astype(np.float32)
    y = ctx.alloc(4 * rows)
    r = ctx.alloc(4 * rows)
    ctx.gen_f32(21, 3, rows, r)
    ctx.call("mlm_q4k_gemv_xs", W, rows, cols, ctx.to_device(x16), ctx.to_device(scale), y, r)
    xtrue = x16.astype(np.float32) * np.repeat(scale, 32)
    ref = O.q4k_matvec_f32x(O.gen_q4k(21, 1, nb), rows, cols, xtrue) + O.gen_f32(21, 3, rows)
    assert rel_l2(y.download(np.float32), ref) < TOL


def test_gemv_rmsnorm_input(ctx):
    """x = fp16(RMSNorm(hidden)) formed inside the GEMV."""
    rows, cols = 6144, 4096
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(23, 1, nb, W)
    h = O.gen_f32(23, 2, cols, 0.0, 3.0)
    w = O.gen_f32(23, 3, cols, 1.0, 0.02)
    y = ctx.alloc(4 * rows)
    ctx.call("mlm_q4k_gemv_rmsnorm", W, rows, cols, ctx.to_device(h), ctx.to_device(w),
             ctypes.c_float(1e-5), y, None)
    xn = O.rmsnorm_f32(h, w, 1, cols, 1e-5).astype(np.float16)
    ref = O.q4k_matvec(O.gen_q4k(23, 1, nb), rows, cols, xn, acc64=True)
    assert rel_l2(y.download(np.float32), ref) < TOL


def test_gemv_swiglu_input(ctx):
    """x = silu(gate) * up formed inside the GEMV (large values: scaled fp16)."""
    rows, cols = 4096, 14336
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(24, 1, nb, W)
    g = O.gen_f32(24, 2, cols, 0.0, 200.0)
    u = O.gen_f32(24, 3, cols, 0.0, 200.0)
    r = O.gen_f32(24, 4, rows)
    y = ctx.alloc(4 * rows)
    ctx.call("mlm_q4k_gemv_swiglu", W, rows, cols, ctx.to_device(g), ctx.to_device(u), y,
             ctx.to_device(r))
    ref = O.q4k_matvec_f32x(O.gen_q4k(24, 1, nb), rows, cols, O.silu_mul(g, u)) + r
    got = y.download(np.float32)
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) < 1e-3  # x rounded to fp16 (2^-11 per element)


@pytest.mark.parametrize("F,cols", [(14336, 4096), (2816, 1024)])
def test_gemv_gate_up_pairs(ctx, F, cols):
    """mlm_q4k_gemv_gate_up over [gate; up] rows: y equals mlm_q4k_gemv_rmsnorm's
    bit for bit, the h / h_scale its epilogue forms equal mlm_silu_mul_scaled
    on that y bit for bit, and the down projection on h (mlm_q4k_gemv_xs)
    equals mlm_q4k_gemv_swiglu on y bit for bit.  Three launches in a row:
    the pairing counters re-zero themselves."""
    rows = 2 * F
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(31, 1, nb, W)
    h = ctx.to_device(O.gen_f32(31, 2, cols, 0.0, 3.0))
    # large norm weights: some sub-blocks of silu(gate) * up pass 2^15 and
    # take a scale above 1
    w = ctx.to_device(O.gen_f32(31, 3, cols, 40.0, 10.0))
    eps = ctypes.c_float(1e-5)
    y_ref = ctx.alloc(4 * rows)
    ctx.call("mlm_q4k_gemv_rmsnorm", W, rows, cols, h, w, eps, y_ref, None)
    hs_ref, sc_ref = ctx.alloc(2 * F), ctx.alloc(4 * (F // 32))
    ctx.call("mlm_silu_mul_scaled", y_ref, int(y_ref) + 4 * F, hs_ref, sc_ref, F)
    want_y = y_ref.download(np.float32)
    want_h = hs_ref.download(np.uint16)
    want_s = sc_ref.download(np.float32)
    assert np.any(want_s > 1.0)
    for _ in range(3):
        y, hs, sc = ctx.alloc(4 * rows), ctx.alloc(2 * F), ctx.alloc(4 * (F // 32))
        ctx.call("mlm_q4k_gemv_gate_up", W, rows, cols, h, w, eps, y, hs, sc)
        assert np.array_equal(y.download(np.float32), want_y)
        assert np.array_equal(hs.download(np.uint16), want_h)
        assert np.array_equal(sc.download(np.float32), want_s)
    # the down projection: staged fp16 h against the SwiGLU staging
    dn = 4096 if cols == 4096 else 1024
    nbd = dn * F // 256
    Wd = ctx.alloc(nbd * 144)
    ctx.gen_q4k(32, 1, nbd, Wd)
    r = ctx.to_device(O.gen_f32(32, 4, dn))
    a, b = ctx.alloc(4 * dn), ctx.alloc(4 * dn)
    ctx.call("mlm_q4k_gemv_xs", Wd, dn, F, hs, sc, a, r)
    ctx.call("mlm_q4k_gemv_swiglu", Wd, dn, F, y_ref, int(y_ref) + 4 * F, b, r)
    assert np.array_equal(a.download(np.float32), b.download(np.float32))
