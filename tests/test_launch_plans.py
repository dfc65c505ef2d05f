"""The decode GEMVs' launch plans, computed on the host (no GPU): the C ABI's
mlm_q4k_gemv_plan / mlm_q4k_gemv_batch_plan.

- Single-token GEMV: whole 32-row tiles per CTA whenever a CTA count
  between half and all of the SMs divides the tiles without raising the
  most units (32x256 blocks) a warp takes; else every SM gets a CTA.
- Batched GEMV: the widest K chunk (block columns) whose grid fills the
  SMs, at most one CTA per SM (one wave).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import metallm_b200._lib as L

SMS = 148  # B200


@pytest.fixture(scope="module")
def lib():
    return L.load()


def gemv_plan(lib, rows, cols, sms=SMS):
    c, w, whole = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    assert lib.mlm_q4k_gemv_plan(rows, cols, sms, ctypes.byref(c), ctypes.byref(w),
                                 ctypes.byref(whole)) == 0
    return c.value, w.value, bool(whole.value)


def batch_plan(lib, rows, cols, sms=SMS):
    ch, c = ctypes.c_int32(), ctypes.c_int32()
    assert lib.mlm_q4k_gemv_batch_plan(rows, cols, sms, ctypes.byref(ch), ctypes.byref(c)) == 0
    return ch.value, c.value


@pytest.mark.parametrize("rows,cols,ctas,whole", [
    (6144, 4096, 96, True),      # 8B QKV: 2 tiles per CTA
    (4096, 4096, 128, True),     # 8B output projection
    (28672, 4096, 128, True),    # 8B gate/up: 7 tiles per CTA
    (4096, 14336, 128, True),    # 8B down
    (14336, 4096, 112, True),    # the headline shape: 4 tiles per CTA
    (8192, 8192, 128, True),     # 70B output projection
    (128256, 4096, 148, False),  # the 8B head: 4008 tiles, no divisor in [74, 148]
    (10240, 8192, 148, False),   # 70B QKV: 80 CTAs would give 8 units a warp, not 5
])
def test_gemv_plans_of_the_model_shapes(lib, rows, cols, ctas, whole):
    c, w, wh = gemv_plan(lib, rows, cols)
    assert (c, wh) == (ctas, whole)
    assert w == 16


def _units_per_warp(units_per_cta, warps):
    return -(-units_per_cta // min(warps, units_per_cta))


def test_whole_tile_plans_never_cost_a_warp_more_units(lib):
    rng = np.random.default_rng(3)
    for _ in range(300):
        tiles = int(rng.integers(1, 5000))
        nb = int(rng.choice([4, 8, 11, 16, 32, 56]))
        rows, cols = tiles * 32, nb * 256
        c, w, whole = gemv_plan(lib, rows, cols)
        units = tiles * nb
        split = min(SMS, units)
        split_cost = _units_per_warp(-(-units // split), w)
        if whole:
            assert tiles % c == 0 and 2 * c >= SMS and c <= SMS
            assert _units_per_warp(tiles // c * nb, w) <= split_cost
        else:
            assert c == split


@pytest.mark.parametrize("rows,cols,chunk,ctas", [
    (10240, 8192, 8, 148),   # 70B QKV, one GPU
    (57344, 8192, 8, 148),   # 70B gate/up
    (8192, 28672, 8, 140),   # 70B down: 14 chunks x 10 (one wave)
    (2560, 8192, 2, 144),    # a rank's QKV at 4 GPUs
    (8192, 2048, 2, 132),    # a rank's output projection at 4 GPUs
    (8192, 7168, 8, 132),    # a rank's down projection at 4 GPUs
])
def test_batch_plans(lib, rows, cols, chunk, ctas):
    assert batch_plan(lib, rows, cols) == (chunk, ctas)


def test_batch_plans_run_in_one_wave(lib):
    for rows in (16, 300, 1000, 2560, 8192, 57344, 128256):
        for cols in (256, 512, 2048, 7168, 8192, 28672):
            chunk, ctas = batch_plan(lib, rows, cols)
            assert chunk in (1, 2, 4, 8)
            assert 1 <= ctas <= SMS, (rows, cols, chunk, ctas)


def test_plans_reject_bad_shapes(lib):
    c = ctypes.c_int32()
    assert lib.mlm_q4k_gemv_plan(128, 300, SMS, ctypes.byref(c), ctypes.byref(c),
                                 ctypes.byref(c)) != 0
    assert lib.mlm_q4k_gemv_batch_plan(0, 256, SMS, ctypes.byref(c), ctypes.byref(c)) != 0
