"""Q6_K and the GGUF Q4_K element order on CPU: the oracle against the
reference's own kernel and against hand-built known-answer blocks.

- Q6_K: orc_q6k_dequant_f32 equals kernel_dequantize_q6_K_f32
  (DequantKernels.metal:131-172) compiled for the host, bit for bit; a block
  encoded by an independent numpy restatement of the layout decodes to the
  values the formula gives.
- Q4_K in the GGUF order: a known-answer block (d = 1, dmin = 0.5,
  sc_j = j + 1, m_j = j, q_i = i mod 16) decodes as specified; the repack to
  the reference's interleaved order, dequantized by the reference's kernel,
  equals the GGUF-order dequant bit for bit, and is a bijection.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O


def _ref_or_skip():
    if O.ref_lib() is None:
        pytest.skip("reference kernels not built (oracle/_ref)")


# -- Q6_K ------------------------------------------------------------------------

def encode_q6k(q6: np.ndarray, scales: np.ndarray, d: float) -> np.ndarray:
    """One 210-byte block from 256 six-bit quants (0..63), 16 int8 scales and
    d: element 128h + 32k + l goes to the low (k < 2) or high nibble of
    ql[64h + l + 32 (k & 1)] and to bits 2k, 2k+1 of qh[32h + l]."""
    ql = np.zeros(128, dtype=np.uint8)
    qh = np.zeros(64, dtype=np.uint8)
    for h in range(2):
        for k in range(4):
            for l in range(32):
                q = int(q6[128 * h + 32 * k + l])
                i = 64 * h + l + 32 * (k & 1)
                ql[i] |= (q & 0xF) << (0 if k < 2 else 4)
                qh[32 * h + l] |= (q >> 4) << (2 * k)
    blk = np.concatenate([ql, qh, scales.astype(np.int8).view(np.uint8),
                          np.array([d], dtype=np.float16).view(np.uint8)])
    assert blk.size == 210
    return blk


def expected_q6k(q6: np.ndarray, scales: np.ndarray, d: float) -> np.ndarray:
    out = np.empty(256, dtype=np.float32)
    d32 = np.float32(np.float16(d))
    for h in range(2):
        for k in range(4):
            for l in range(32):
                e = 128 * h + 32 * k + l
                s = np.float32(scales[8 * h + 2 * k + l // 16])
                out[e] = np.float32(d32 * s) * np.float32(int(q6[e]) - 32)
    return out


def test_q6k_known_answer_block():
    q6 = (np.arange(256) * 7) % 64
    scales = np.arange(16) - 8
    blk = encode_q6k(q6, scales, 0.5)
    want = expected_q6k(q6, scales, 0.5)
    got = O.q6k_dequant_f32(blk, 256)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("nblocks", [1, 3, 257])
def test_q6k_oracle_matches_reference_kernel(nblocks):
    _ref_or_skip()
    b = O.gen_q6k(17, 4, nblocks)
    a = O.q6k_dequant_f32(b, nblocks * 256)
    r = O.ref_q6k_dequant_f32(b, nblocks * 256, 2)
    assert np.array_equal(a.view(np.uint32), r.view(np.uint32))


def test_q6k_generator_fields():
    b = O.gen_q6k(3, 1, 64).reshape(64, 210)
    d = b[:, 208:210].copy().view(np.float16).astype(np.float32).ravel()
    assert np.all(d >= 0) and 0.001 < d.mean() < 0.02  # |N(0,1)| * 0.01
    sc = b[:, 192:208].view(np.int8)
    assert sc.min() < -100 and sc.max() > 100  # uniform int8 scales
    b2 = O.gen_q6k(3, 1, 60, first_block=4).reshape(60, 210)
    assert np.array_equal(b[4:], b2)


def test_q6k_matvec_is_dequant_dot():
    rows, cols = 8, 512
    W = O.gen_q6k(5, 2, rows * cols // 256)
    x = O.gen_f16(5, 3, cols)
    y = O.q6k_matvec(W, rows, cols, x)
    dense = O.q6k_dequant_f32(W, rows * cols).reshape(rows, cols).astype(np.float64)
    want = dense @ x.astype(np.float64)
    assert np.allclose(y, want, rtol=1e-6, atol=1e-5)


# -- Q4_K in the GGUF element order ------------------------------------------------

def encode_q4k_canonical(q: np.ndarray, sc: np.ndarray, m: np.ndarray, d: float,
                         dmin: float) -> np.ndarray:
    """A GGUF-order Q4_K block; scales/mins below 16 so the 12-byte packing is
    s[j] = sc_j, s[j+4] = m_j (j < 4) and s[8+j-4] = sc_j | m_j << 4 (j >= 4)."""
    assert sc.max() < 16 and m.max() < 16
    s = np.zeros(12, dtype=np.uint8)
    for j in range(4):
        s[j] = sc[j]
        s[j + 4] = m[j]
        s[8 + j] = sc[j + 4] | (m[j + 4] << 4)
    qs = np.zeros(128, dtype=np.uint8)
    for i in range(256):
        j, l = divmod(i, 64)
        if l < 32:
            qs[32 * j + l] |= q[i]
        else:
            qs[32 * j + l - 32] |= q[i] << 4
    hdr = np.array([d, dmin], dtype=np.float16).view(np.uint8)
    return np.concatenate([hdr, s, qs])


def test_q4k_canonical_known_answer_block():
    q = np.arange(256) % 16
    sc = np.arange(8) + 1
    m = np.arange(8)
    blk = encode_q4k_canonical(q, sc, m, 1.0, 0.5)
    want = np.array([np.float32(sc[i // 32]) * np.float32(q[i]) - np.float32(0.5 * m[i // 32])
                     for i in range(256)], dtype=np.float32)
    got = O.q4k_dequant_canonical_f32(blk, 256)
    assert np.array_equal(got, want)


def test_q4k_repack_equals_canonical_dequant():
    b = O.gen_q4k(11, 6, 300)
    inter = O.q4k_canonical_to_interleaved(b)
    want = O.q4k_dequant_canonical_f32(b, 300 * 256)
    got = O.q4k_dequant_f32(inter, 300 * 256)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    if O.ref_lib() is not None:  # the reference's own kernel reads the repacked blocks
        r = O.ref_q4k_dequant_f32(inter, 300 * 256, 2)
        assert np.array_equal(r.view(np.uint32), want.view(np.uint32))


def test_q4k_repack_is_a_bijection():
    b = O.gen_q4k(12, 7, 50)
    inter = O.q4k_canonical_to_interleaved(b).reshape(50, 144)
    assert np.array_equal(inter[:, :16], b.reshape(50, 144)[:, :16])  # headers untouched
    # invert: interleaved element i is nibble i % 2 of byte i // 2
    qs = inter[:, 16:]
    nib = np.stack([qs & 0xF, qs >> 4], axis=-1).reshape(50, 256)
    back = np.zeros((50, 128), dtype=np.uint8)
    for i in range(256):
        j, l = divmod(i, 64)
        if l < 32:
            back[:, 32 * j + l] |= nib[:, i]
        else:
            back[:, 32 * j + l - 32] |= nib[:, i] << 4
    assert np.array_equal(back, b.reshape(50, 144)[:, 16:])


def test_q6k_matvec_matches_reference_dequant_dot():
    """The Q6_K matvec oracle against rows dequantized by the reference's own
    kernel_dequantize_q6_K_f32 (what the reference hands to MPS), fp64 dot."""
    _ref_or_skip()
    rows, cols = 24, 2048
    W = O.gen_q6k(13, 2, rows * cols // 256)
    x = O.gen_f16(13, 3, cols)
    dense = O.ref_q6k_dequant_f32(W, rows * cols, 2).reshape(rows, cols).astype(np.float64)
    want = dense @ x.astype(np.float64)
    got = O.q6k_matvec(W, rows, cols, x)
    # both fp64 sums of the same exact products, rounded once to fp32: only
    # the summation order differs
    assert np.allclose(got, want, rtol=1e-6, atol=1e-6)
