"""CPU tests of the oracle: pinned against the reference's own kernels.

The golden vectors were produced by the reference's Metal kernels compiled
for the host (tests/golden/make_golden.py); when oracle/_ref is present the
restatement is also compared with it on fresh seeded inputs.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import rel_l2


def test_generators_deterministic():
    a = O.gen_q4k(1, 2, 100)
    b = O.gen_q4k(1, 2, 100)
    assert np.array_equal(a, b)
    # a sub-range regenerates the same bytes (counter-based)
    c = O.gen_q4k(1, 2, 10, first_block=40)
    assert np.array_equal(a[40 * 144:50 * 144], c)
    # header fields are |N(0,1)| * 0.01 in fp16; payload bytes look uniform
    d = a.reshape(100, 144)[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    assert np.all(d >= 0) and 0.002 < d.mean() < 0.02
    payload = a.reshape(100, 144)[:, 4:].ravel()
    assert 100 < payload.mean() < 155


def test_normal_moments():
    x = O.gen_f32(3, 4, 200_000).astype(np.float64)
    assert abs(x.mean()) < 0.01
    assert abs(x.std() - 1.0) < 0.01


def test_dequant_f32_matches_reference_kernel_golden(golden):
    blocks = golden["q4k_blocks"]
    n = golden["q4k_f32"].size
    out = O.q4k_dequant_f32(blocks, n)
    assert np.array_equal(out.view(np.uint32), golden["q4k_f32"].view(np.uint32))


def test_dequant_f32_ragged_golden(golden):
    n = int(golden["q4k_ragged_n"][0])
    out = O.q4k_dequant_f32(golden["q4k_blocks"], n)
    assert np.array_equal(out.view(np.uint32), golden["q4k_ragged_f32"].view(np.uint32))


def test_dequant_f16_matches_reference_kernel_golden(golden):
    blocks = golden["q4k_blocks"]
    n = golden["q4k_f16"].size
    out = O.q4k_dequant_f16(blocks, n)
    assert np.array_equal(out.view(np.uint16), golden["q4k_f16"].view(np.uint16))


def test_dequant_known_answer_block(golden):
    # block 66 (64 seeded + edge block #2): d=1, dmin=0.5, sc_j=j+1, m_j=j, q_i=i%16
    out = O.q4k_dequant_f32(golden["q4k_blocks"], golden["q4k_f32"].size).reshape(-1, 256)[66]
    i = np.arange(256)
    j = i // 32
    expect = (j + 1) * (i % 16) - 0.5 * j
    assert np.array_equal(out, expect.astype(np.float32))
    # edge block #1: all nibbles 15 and sc = m = 63: 1*63*15 - 0.5*63
    out1 = O.q4k_dequant_f32(golden["q4k_blocks"], golden["q4k_f32"].size).reshape(-1, 256)[65]
    assert np.all(out1 == np.float32(63 * 15 - 0.5 * 63))
    # edge block #0: all zero
    out0 = O.q4k_dequant_f32(golden["q4k_blocks"], golden["q4k_f32"].size).reshape(-1, 256)[64]
    assert np.all(out0 == 0)


def test_scale_min_unpack_exhaustive_bytes():
    """get_scale_min_k4 restated vs a direct bit-level reading of the packing."""
    rng = np.random.default_rng(0)
    for _ in range(200):
        s = rng.integers(0, 256, 12, dtype=np.uint8)
        for j in range(8):
            if j < 4:
                sc, m = s[j] & 63, s[j + 4] & 63
            else:
                sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4)
                m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4)
            blk = np.zeros(144, dtype=np.uint8)
            blk[0:2] = np.array([1.0], dtype=np.float16).view(np.uint8)
            blk[2:4] = np.array([1.0], dtype=np.float16).view(np.uint8)
            blk[4:16] = s
            blk[16:] = 0x11  # every q = 1
            out = O.q4k_dequant_f32(blk, 256)
            assert out[32 * j] == np.float32(sc) - np.float32(m)


def test_matvec_golden(golden):
    rows, cols = (int(v) for v in golden["mv_shape"])
    y = O.q4k_matvec(golden["mv_W"], rows, cols, golden["mv_x"], acc64=True)
    # the golden y accumulates in fp32 in the reference's order; the oracle in fp64
    assert rel_l2(y, golden["mv_y"]) < 1e-6


def test_rmsnorm_golden(golden):
    rr, nn = (int(v) for v in golden["rms_shape"])
    y = O.rmsnorm_f16(golden["rms_x"], golden["rms_w"], rr, nn, float(golden["rms_eps"][0]))
    d = np.abs(y.view(np.int16).astype(np.int32) - golden["rms_y"].view(np.int16).astype(np.int32))
    assert d.max() <= 1  # sum-of-squares order only
    assert np.mean(d == 0) > 0.99


@pytest.mark.parametrize("pos", [0, 2047])
def test_rope_golden(golden, pos):
    seq, heads, d = (int(v) for v in golden["rope_shape"])
    out = O.rope_f16(O.rope_args(pos_offset=pos), golden["rope_in"], seq, heads, d)
    assert np.array_equal(out.view(np.uint16), golden[f"rope_out_pos{pos}"].view(np.uint16))


def test_rope_yarn_golden(golden):
    seq, heads, d = (int(v) for v in golden["rope_shape"])
    a = O.rope_args(pos_offset=1000, ext_factor=1.0, freq_scale=0.25, n_ctx_orig=8192,
                    has_freq_factors=True)
    out = O.rope_f16(a, golden["rope_in"], seq, heads, d, golden["rope_freqs"])
    ref = golden["rope_out_yarn"]
    diff = np.abs(out.astype(np.float32) - ref.astype(np.float32))
    assert diff.max() <= 2e-3


def test_attention_decode_properties():
    # softmax over one position returns V; identical keys average V
    d, nkv, nh = 128, 2, 4
    q = O.gen_f32(1, 1, nh * d)
    k = O.gen_f16(1, 2, 1 * nkv * d)
    v = O.gen_f16(1, 3, 1 * nkv * d)
    out = O.attn_decode(q, k, v, nh, nkv, d, 1).reshape(nh, d)
    vv = v.reshape(1, nkv, d).astype(np.float32)
    for h in range(nh):
        assert np.allclose(out[h], vv[0, h // 2], atol=1e-6)
    k2 = np.tile(k.reshape(1, nkv * d), (5, 1)).ravel()
    v2 = O.gen_f16(1, 4, 5 * nkv * d)
    out2 = O.attn_decode(q, k2, v2, nh, nkv, d, 5).reshape(nh, d)
    vm = v2.reshape(5, nkv, d).astype(np.float64).mean(axis=0)
    for h in range(nh):
        assert np.allclose(out2[h], vm[h // 2], atol=1e-5)


@pytest.mark.skipif(O.ref_lib() is None, reason="reference kernels not built (make -C oracle ref)")
class TestAgainstReferenceKernels:
    """Fresh seeded inputs through both the restatement and the reference."""

    def test_dequant_f32_config0_blocks(self):
        nb = 65536  # 4096 x 4096 weight, the CPU-vs-GPU dequant workload
        W = O.gen_q4k(1234, 0, nb)
        a = O.q4k_dequant_f32(W, nb * 256)
        b = O.ref_q4k_dequant_f32(W, nb * 256, 8)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))

    def test_dequant_f16(self):
        W = O.gen_q4k(99, 1, 4096)
        a = O.q4k_dequant_f16(W, 4096 * 256)
        b = O.ref_q4k_dequant_f16(W, 4096 * 256, 8)
        assert np.array_equal(a.view(np.uint16), b.view(np.uint16))

    def test_rope_positions(self):
        q = O.gen_f16(3, 1, 4 * 32 * 128)
        for pos in (1, 511, 8191):
            a = O.rope_args(pos_offset=pos)
            x = O.rope_f16(a, q, 4, 32, 128)
            y = O.ref_rope_f16(a, q, 4, 32)
            assert np.array_equal(x.view(np.uint16), y.view(np.uint16))

    def test_matvec(self):
        rows, cols = 64, 2048
        W = O.gen_q4k(5, 5, rows * cols // 256)
        x = O.gen_f16(5, 6, cols)
        assert rel_l2(O.ref_q4k_matvec(W, rows, cols, x, 4), O.q4k_matvec(W, rows, cols, x)) < 1e-6
