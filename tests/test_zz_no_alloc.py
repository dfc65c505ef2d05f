"""mlm_q4k_gemv_static (split-K scratch in a static device array, no
allocation) against mlm_q4k_gemv, through the C ABI.

Kept in a file of its own that collects last, so it runs both after the
other GPU tests (the array then holds whatever earlier calls left) and
alone in a fresh process (the first call does the per-device set-up).
Bar: the GEMV tolerance, relative L2 <= 1e-5, on two calls in a row.
"""
from __future__ import annotations

import numpy as np
import pytest

from metallm_b200 import MLMError
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-5
MAX_ROWS = 131072


def _static(ctx, W, rows, cols, x, y, r=None):
    ctx.call("mlm_q4k_gemv_static", W, rows, cols, x, y, r)


@pytest.mark.parametrize("rows,cols", [
    (14336, 4096),    # FFN up/gate: tiles split across CTAs
    (4096, 14336),    # FFN down
    (32, 14336),      # one row tile shared by every CTA
    (100, 512),       # ragged last tile
    (MAX_ROWS, 256),  # the row limit, one block per row
])
def test_static_matches_gemv_two_calls(ctx, rows, cols):
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(31, 1, nb, W)
    xs = [ctx.alloc(2 * cols) for _ in range(2)]
    for i, x in enumerate(xs):
        ctx.gen_f16(31, 10 + i, cols, x)
    r = ctx.alloc(4 * rows)
    ctx.gen_f32(31, 20, rows, r)
    y_ref = ctx.alloc(4 * rows)
    y_st = ctx.alloc(4 * rows)
    # call 1 without and call 2 with the residual, back to back on the stream
    for i, res in enumerate([None, r]):
        ctx.q4k_gemv(W, rows, cols, xs[i], y_ref, res)
        _static(ctx, W, rows, cols, xs[i], y_st, res)
        want = y_ref.download(np.float32)
        got = y_st.download(np.float32)
        assert np.all(np.isfinite(got)), (rows, cols, i)
        assert rel_l2(got, want) <= TOL, (rows, cols, i)


def test_static_allocates_nothing(ctx):
    """After the per-device set-up, calls leave the device's free memory
    unchanged (cudaMemGetInfo before and after several calls)."""
    import torch
    rows, cols = 14336, 4096
    nb = rows * cols // 256
    W = ctx.alloc(nb * 144)
    ctx.gen_q4k(33, 1, nb, W)
    x = ctx.alloc(2 * cols)
    ctx.gen_f16(33, 2, cols, x)
    y = ctx.alloc(4 * rows)
    torch.cuda.mem_get_info(ctx.device)  # torch's own lazy set-up, outside the window
    _static(ctx, W, rows, cols, x, y)
    ctx.wait()
    free0, _ = torch.cuda.mem_get_info(ctx.device)
    for _ in range(4):
        _static(ctx, W, rows, cols, x, y)
    ctx.wait()
    free1, _ = torch.cuda.mem_get_info(ctx.device)
    assert free1 == free0, (free0, free1)


def test_static_rejects_rows_beyond_limit(ctx):
    cols = 256
    W = ctx.alloc(144 * 4)
    x = ctx.alloc(2 * cols)
    y = ctx.alloc(16)
    with pytest.raises(MLMError) as e:
        _static(ctx, W, MAX_ROWS + 1, cols, x, y)
    assert e.value.status == -2
    assert "static scratch limit" in str(e.value)
