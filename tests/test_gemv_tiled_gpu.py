"""The tiled Q4_K layout and the GEMV on it, through the C ABI.

The layout is checked byte for byte against a numpy restatement; the GEMV
against the oracle's fp64 product of the bit-exact fp32 dequantization
(relative L2 <= 1e-5, the GGUF-layout GEMV's bar).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-5


def tile_reference(blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Unit (t, b) = [headers [i][g] | quants [i][h][g][t]], 16-byte pieces."""
    nb = cols // 256
    T = (rows + 31) // 32
    pad = np.zeros((T * 32, nb, 144), dtype=np.uint8)
    pad[:rows] = blocks.reshape(rows, nb, 144)
    P = pad.reshape(T, 4, 8, nb, 144)                       # [t][i][g][b][byte]
    hdr = P[..., :16].transpose(0, 3, 1, 2, 4).reshape(T, nb, 512)
    q = P[..., 16:].reshape(T, 4, 8, nb, 2, 4, 16)          # [t][i][g][b][h][t'][16]
    q = q.transpose(0, 3, 1, 4, 2, 5, 6).reshape(T, nb, 4096)
    return np.concatenate([hdr, q], axis=-1).reshape(-1)


def _tiled(ctx, W, rows, cols):
    Wt = ctx.alloc(ctx.q4k_tiled_bytes(rows, cols))
    ctx.q4k_tile(W, rows, cols, Wt)
    return Wt


@pytest.mark.parametrize("rows,cols", [(32, 256), (40, 512), (1, 256), (100, 768)])
def test_tile_layout(ctx, rows, cols):
    nb = rows * cols // 256
    blocks = O.gen_q4k(5, 1, nb)
    W = ctx.to_device(blocks)
    Wt = _tiled(ctx, W, rows, cols)
    got = Wt.download(np.uint8)[: ctx.q4k_tiled_bytes(rows, cols)]
    np.testing.assert_array_equal(got, tile_reference(blocks, rows, cols))


def test_tiled_bytes(ctx):
    assert ctx.q4k_tiled_bytes(14336, 4096) == 14336 * 16 * 144
    assert ctx.q4k_tiled_bytes(33, 256) == 64 * 144
    assert ctx.q4k_tiled_bytes(10, 300) == 0


def _run(ctx, rows, cols, seed=11, residual=False):
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(seed, 1, nb, W)
    Wt = _tiled(ctx, W, rows, cols)
    x = ctx.alloc(2 * cols)
    ctx.gen_f16(seed, 2, cols, x)
    y = ctx.alloc(4 * rows)
    r = None
    if residual:
        r = ctx.alloc(4 * rows)
        ctx.gen_f32(seed, 3, rows, r)
    ctx.q4k_gemv_tiled(Wt, rows, cols, x, y, r)
    got = y.download(np.float32)
    ref = O.q4k_matvec(O.gen_q4k(seed, 1, nb), rows, cols, O.gen_f16(seed, 2, cols), acc64=True)
    if residual:
        ref = ref + O.gen_f32(seed, 3, rows)
    return got, ref


def test_gemv_tiled_golden(ctx, golden):
    rows, cols = (int(v) for v in golden["mv_shape"])
    W = ctx.to_device(golden["mv_W"])
    Wt = _tiled(ctx, W, rows, cols)
    x = ctx.to_device(golden["mv_x"])
    y = ctx.alloc(4 * rows)
    ctx.q4k_gemv_tiled(Wt, rows, cols, x, y)
    assert rel_l2(y.download(np.float32), golden["mv_y"]) < TOL


@pytest.mark.parametrize("rows,cols", [(256, 256), (16, 256), (1, 512), (100, 512), (33, 4096),
                                       (4096, 4096), (1024, 14336), (3000, 768), (14336, 4096),
                                       (4096, 14336), (32, 14336), (128256, 256)])
def test_gemv_tiled_shapes(ctx, rows, cols):
    got, ref = _run(ctx, rows, cols)
    assert np.all(np.isfinite(got))
    assert rel_l2(got, ref) < TOL, (rows, cols)


def test_gemv_tiled_residual(ctx):
    got, ref = _run(ctx, 777, 2048, residual=True)
    assert rel_l2(got, ref) < TOL


def test_gemv_tiled_deterministic_and_graph(ctx):
    rows, cols = 14336, 4096
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(3, 1, nb, W)
    Wt = _tiled(ctx, W, rows, cols)
    x = ctx.alloc(2 * cols)
    ctx.gen_f16(3, 2, cols, x)
    y0, y1 = ctx.alloc(4 * rows), ctx.alloc(4 * rows)
    ctx.q4k_gemv_tiled(Wt, rows, cols, x, y0)
    a = y0.download(np.float32)
    ctx.graph_begin()
    for _ in range(3):
        ctx.q4k_gemv_tiled(Wt, rows, cols, x, y1)
    g = ctx.graph_end()
    g.launch()
    ctx.wait()
    np.testing.assert_array_equal(y1.download(np.float32), a)
    g.destroy()


def test_gemv_tiled_bad_args(ctx):
    from metallm_b200 import MLMError
    W = ctx.alloc(144 * 64)
    x = ctx.alloc(2 * 512)
    y = ctx.alloc(4 * 32)
    with pytest.raises(MLMError) as e:
        ctx.q4k_gemv_tiled(W, 2, 300, x, y)
    assert e.value.status == -2
    with pytest.raises(MLMError) as e:
        ctx.q4k_gemv_tiled(W.ptr + 8, 2, 256, x, y)
    assert e.value.status == -3
    with pytest.raises(MLMError) as e:
        ctx.q4k_tile(W, 2, 300, W)
    assert e.value.status == -2
