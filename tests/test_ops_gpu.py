"""GPU parity of RMSNorm, RoPE, decode attention and the small ops."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from metallm_b200 import rope_args
from oracle import oracle as O
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu


def _ulp16(a, b):
    return np.abs(a.view(np.int16).astype(np.int32) - b.view(np.int16).astype(np.int32))


def test_rmsnorm_f16_golden(ctx, golden):
    rr, nn = (int(v) for v in golden["rms_shape"])
    x = ctx.to_device(golden["rms_x"])
    w = ctx.to_device(golden["rms_w"])
    y = ctx.alloc(2 * rr * nn)
    ctx.call("mlm_rmsnorm_f16", x, w, y, rr, nn, ctypes.c_float(float(golden["rms_eps"][0])))
    got = y.download(np.float16)
    d = _ulp16(got, golden["rms_y"])
    assert d.max() <= 1 and np.mean(d == 0) > 0.99  # summation order only


def test_rmsnorm_f32_layer_input(ctx):
    n = 4096
    x = O.gen_f32(3, 1, n)
    w = O.gen_f32(3, 2, n, mean=1.0, std=0.02)
    dx, dw = ctx.to_device(x), ctx.to_device(w)
    y32, y16 = ctx.alloc(4 * n), ctx.alloc(2 * n)
    ctx.call("mlm_rmsnorm_f32", dx, dw, y32, y16, 1, n, ctypes.c_float(1e-5))
    ref = O.rmsnorm_f32(x, w, 1, n, 1e-5)
    assert rel_l2(y32.download(np.float32), ref) < 1e-6
    assert np.array_equal(y16.download(np.float16),
                          y32.download(np.float32).astype(np.float16))


def test_rmsnorm_tiny_input_clamps(ctx):
    # mean(x^2) below 1e-10 uses the floor, and the 1e6 cap
    n = 256
    x = np.full(n, 1e-7, dtype=np.float32)
    w = np.ones(n, dtype=np.float32)
    y32 = ctx.alloc(4 * n)
    ctx.call("mlm_rmsnorm_f32", ctx.to_device(x), ctx.to_device(w), y32, None, 1, n,
             ctypes.c_float(0.0))
    ref = O.rmsnorm_f32(x, w, 1, n, 0.0)
    assert np.allclose(y32.download(np.float32), ref, rtol=1e-6)


@pytest.mark.parametrize("pos", [0, 2047])
def test_rope_f16_golden(ctx, golden, pos):
    seq, heads, d = (int(v) for v in golden["rope_shape"])
    buf = ctx.to_device(golden["rope_in"])
    a = rope_args(pos_offset=pos)
    ctx.call("mlm_rope_f16", buf, None, ctypes.byref(a), seq, heads, d)
    got = buf.download(np.float16)
    ref = golden[f"rope_out_pos{pos}"]
    d16 = _ulp16(got, ref)
    assert d16.max() <= 1 and np.mean(d16 == 0) > 0.995


def test_rope_f16_yarn_freq_factors(ctx, golden):
    seq, heads, d = (int(v) for v in golden["rope_shape"])
    buf = ctx.to_device(golden["rope_in"])
    ff = ctx.to_device(golden["rope_freqs"])
    a = rope_args(pos_offset=1000, ext_factor=1.0, freq_scale=0.25, n_ctx_orig=8192,
                  has_freq_factors=True)
    ctx.call("mlm_rope_f16", buf, ff, ctypes.byref(a), seq, heads, d)
    got = buf.download(np.float16).astype(np.float32)
    assert np.abs(got - golden["rope_out_yarn"].astype(np.float32)).max() <= 2e-3


def test_rope_qk_kv_append(ctx):
    nq, nkv, d, pos, maxseq = 32, 8, 128, 2047, 2048
    q = O.gen_f32(4, 1, nq * d)
    k = O.gen_f32(4, 2, nkv * d)
    v = O.gen_f32(4, 3, nkv * d)
    dq, dk, dv = ctx.to_device(q), ctx.to_device(k), ctx.to_device(v)
    qo = ctx.alloc(2 * nq * d)
    kc = ctx.alloc(2 * maxseq * nkv * d)
    vc = ctx.alloc(2 * maxseq * nkv * d)
    a = rope_args(pos_offset=pos)
    ctx.call("mlm_rope_qk_kv_append", dq, dk, dv, None, ctypes.byref(a), nq, nkv, d, qo, kc, vc,
             pos)
    oa = O.rope_args(pos_offset=pos)
    rq = O.rope_f32(oa, q, 1, nq, d)
    rk = O.rope_f32(oa, k, 1, nkv, d)
    assert rel_l2(qo.download(np.float16).astype(np.float32), rq) < 1e-3
    kcache = kc.download(np.float16).reshape(maxseq, nkv * d)
    vcache = vc.download(np.float16).reshape(maxseq, nkv * d)
    assert rel_l2(kcache[pos].astype(np.float32), rk) < 1e-3
    assert np.array_equal(vcache[pos], v.astype(np.float16))


@pytest.mark.parametrize("nh,nkv,seq", [(32, 8, 2048), (32, 8, 1), (32, 8, 77), (64, 8, 2176),
                                        (8, 8, 300), (16, 8, 5000)])
def test_attn_decode(ctx, nh, nkv, seq):
    d = 128
    qf = O.gen_f32(6, 1, nh * d)
    q16 = qf.astype(np.float16)
    kc = O.gen_f16(6, 2, seq * nkv * d)
    vc = O.gen_f16(6, 3, seq * nkv * d)
    out = ctx.alloc(2 * nh * d)
    ctx.call("mlm_attn_decode", ctx.to_device(q16), ctx.to_device(kc), ctx.to_device(vc), nh,
             nkv, d, seq, out)
    ref = O.attn_decode(q16.astype(np.float32), kc, vc, nh, nkv, d, seq)
    assert rel_l2(out.download(np.float16).astype(np.float32), ref) < 2e-3


def test_silu_mul_and_add(ctx):
    n = 14336
    g = O.gen_f32(8, 1, n, std=3.0)
    u = O.gen_f32(8, 2, n)
    out = ctx.alloc(2 * n)
    ctx.call("mlm_silu_mul", ctx.to_device(g), ctx.to_device(u), out, n)
    ref = O.silu_mul(g, u)
    assert rel_l2(out.download(np.float16).astype(np.float32), ref) < 1e-3
    s = ctx.alloc(4 * n)
    ctx.call("mlm_add_f32", ctx.to_device(g), ctx.to_device(u), s, n)
    assert np.array_equal(s.download(np.float32), g + u)


def test_argmax_first_max_and_embed(ctx):
    n = 128256
    x = O.gen_f32(1, 1, n)
    x[5000] = 10.0
    x[90000] = 10.0
    x[7] = np.nan
    idx = ctx.alloc(16)
    ctx.call("mlm_argmax_f32", ctx.to_device(x), n, idx)
    assert idx.download(np.int32, 1)[0] == 5000
    vocab, dim = 1000, 4096
    table = O.gen_f16(2, 5, vocab * dim, std=0.02)
    tok = ctx.to_device(np.array([321], dtype=np.int32))
    out = ctx.alloc(4 * dim)
    ctx.call("mlm_embed_f16", ctx.to_device(table), vocab, dim, tok, out)
    assert np.array_equal(out.download(np.float32),
                          table.reshape(vocab, dim)[321].astype(np.float32))


def _argmax_ref(x: np.ndarray) -> int:
    """First index of the maximum with NaN never winning; all-NaN -> 0."""
    v = np.where(np.isnan(x), -np.inf, x)
    if np.all(np.isnan(x)):
        return 0
    m = v.max()
    if m == -np.inf:  # only -inf and NaN: the first -inf
        return int(np.nonzero(x == -np.inf)[0][0])
    return int(np.argmax(v == m))


@pytest.mark.parametrize("n", [1, 7, 1000, 4097, 128256, 1 << 20])
def test_argmax_sizes_ties_nan(ctx, n):
    """Device-wide argmax over several CTAs: ties resolve to the first index,
    NaN never wins, negative values and -inf order correctly; repeated calls
    (the running key is reset by the last CTA of each call)."""
    rng = np.random.default_rng(n)
    idx = ctx.alloc(16)
    cases = [rng.standard_normal(n).astype(np.float32) - 5.0]
    x = rng.standard_normal(n).astype(np.float32)
    x[rng.integers(0, n, size=max(1, n // 50))] = np.nan
    if n > 3:
        x[n - 2] = x[n // 3] = np.float32(50.0)  # tie: the earlier index wins
    cases.append(x)
    cases.append(np.full(n, np.nan, dtype=np.float32))
    y = np.full(n, -np.inf, dtype=np.float32)
    y[: n // 2] = np.nan
    cases.append(y)
    for x in cases:
        for _ in range(2):
            ctx.call("mlm_argmax_f32", ctx.to_device(x), n, idx)
            assert int(idx.download(np.int32, 1)[0]) == _argmax_ref(x)


def test_silu_mul_scaled(ctx):
    """fp16 x per-32 power-of-two scale: finite where plain fp16 overflows,
    and equal to the fp16 rounding of the scaled product."""
    n = 14336
    g = O.gen_f32(41, 1, n, 0.0, 300.0)
    u = O.gen_f32(41, 2, n, 0.0, 300.0)
    gd, ud = ctx.to_device(g), ctx.to_device(u)
    out, sc = ctx.alloc(2 * n), ctx.alloc(4 * (n // 32))
    ctx.call("mlm_silu_mul_scaled", gd, ud, out, sc, n)
    h16 = out.download(np.float16)[:n]
    s = sc.download(np.float32)[: n // 32]
    ref = O.silu_mul(g, u).astype(np.float64)
    assert np.all(np.isfinite(h16))
    assert np.any(np.abs(ref) > 65504.0)  # the case a plain fp16 store overflows
    e = np.log2(s)
    assert np.all(e == np.round(e)) and np.all(e >= 0)
    blocks = np.abs(h16.astype(np.float32)).reshape(-1, 32).max(axis=1)
    assert np.all(blocks <= 32768.0)  # fp16 rounding may reach 2^15 exactly
    got = h16.astype(np.float64) * np.repeat(s, 32)
    # fp16 rounding of the scaled value: half an ulp, or the subnormal spacing
    # 2^-24 (times the scale) near zero
    bound = np.maximum(2.0 ** -11 * np.abs(ref), 2.0 ** -24 * np.repeat(s, 32))
    assert np.all(np.abs(got - ref) <= bound)
