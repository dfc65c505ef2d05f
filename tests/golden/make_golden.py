"""Generate the golden vectors under tests/golden/ from the reference itself.

The outputs come from the reference's own Metal kernels
(MetalLM/Backend/Metal/*.metal) compiled as host C++ by ``make -C oracle ref``
and executed on the CPU through oracle/_ref/libmetal_ref.so.  The inputs are
seeded synthetic data from the oracle generators plus hand-built edge blocks.

    make -C oracle ref && python tests/golden/make_golden.py

Only needed when the fixtures change; the tests read the committed .npz.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")


def half_bits(v: float) -> int:
    return int(np.array([v], dtype=np.float16).view(np.uint16)[0])


def edge_blocks() -> np.ndarray:
    """Hand-built super-blocks covering the corners of the format."""
    blocks = []

    def blk(d, dmin, scales: bytes, qs: bytes) -> np.ndarray:
        b = np.zeros(144, dtype=np.uint8)
        b[0:2] = np.array([half_bits(d)], dtype=np.uint16).view(np.uint8)
        b[2:4] = np.array([half_bits(dmin)], dtype=np.uint16).view(np.uint8)
        b[4:16] = np.frombuffer(scales, dtype=np.uint8)
        b[16:144] = np.frombuffer(qs, dtype=np.uint8)
        return b

    # all zero
    blocks.append(blk(0.0, 0.0, bytes(12), bytes(128)))
    # all nibbles 15, all scale/min bits set (sc = m = 63 everywhere)
    blocks.append(blk(1.0, 0.5, bytes([0xFF] * 12), bytes([0xFF] * 128)))
    # known answer: d = 1, dmin = 0.5, sc_j = j + 1, m_j = j, q_i = i % 16
    sc = list(range(1, 9))
    mn = list(range(0, 8))
    s = [0] * 12
    for j in range(4):
        s[j] = sc[j] | ((sc[j + 4] >> 4) << 6)
        s[j + 4] = mn[j] | ((mn[j + 4] >> 4) << 6)
        s[j + 8] = (sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4)
    qs = bytes(((2 * p) % 16) | (((2 * p + 1) % 16) << 4) for p in range(128))
    blocks.append(blk(1.0, 0.5, bytes(s), qs))
    # scale bytes whose high bits feed sub-blocks 4..7
    blocks.append(blk(0.25, 0.125, bytes([0xC0, 0x80, 0x40, 0xC3, 0xC1, 0x3F, 0x81, 0x7E,
                                          0x0F, 0xF0, 0xA5, 0x5A]), bytes(range(128))))
    # subnormal fp16 d and dmin
    blocks.append(blk(2.0 ** -24 * 3, 2.0 ** -20, bytes([0x55] * 12), bytes([0xA7] * 128)))
    # largest finite fp16 d, negative d and dmin
    blocks.append(blk(65504.0, -2.0, bytes([0x3F] * 12), bytes([0x5A] * 128)))
    blocks.append(blk(-0.0078125, -0.001, bytes([0x12, 0x34, 0x56, 0x78, 0x9A, 0xBC, 0xDE,
                                                  0xF0, 0x11, 0x22, 0x33, 0x44]),
                      bytes([0x0F] * 64 + [0xF0] * 64)))
    return np.concatenate(blocks)


def main() -> None:
    if O.ref_lib() is None:
        raise SystemExit("oracle/_ref/libmetal_ref.so missing: run `make -C oracle ref`")
    g = {}
    # --- Q4_K dequant: 64 seeded blocks + edge blocks -------------------------
    seeded = O.gen_q4k(seed=20240501, stream=7, nblocks=64)
    blocks = np.concatenate([seeded, edge_blocks()])
    nb = blocks.size // 144
    n = nb * 256
    g["q4k_blocks"] = blocks
    g["q4k_f32"] = O.ref_q4k_dequant_f32(blocks, n)
    g["q4k_f16"] = O.ref_q4k_dequant_f16(blocks, n)
    # ragged element count (not a multiple of 256)
    g["q4k_ragged_n"] = np.array([n - 77], dtype=np.int64)
    g["q4k_ragged_f32"] = O.ref_q4k_dequant_f32(blocks, n - 77)

    # --- matvec: dequantized by the reference kernel, fp32 dot ----------------
    rows, cols = 48, 1024
    W = O.gen_q4k(seed=77, stream=3, nblocks=rows * cols // 256)
    x = O.gen_f16(seed=77, stream=4, n=cols)
    g["mv_W"] = W
    g["mv_x"] = x
    g["mv_shape"] = np.array([rows, cols], dtype=np.int64)
    g["mv_y"] = O.ref_q4k_matvec(W, rows, cols, x, 1)

    # --- RMSNorm (kernel_rms_norm_f16) -----------------------------------------
    rr, nn = 3, 4096
    xr = O.gen_f16(seed=5, stream=1, n=rr * nn)
    wr = O.gen_f16(seed=5, stream=2, n=nn, mean=1.0, std=0.02)
    wr[17] = np.float16(np.nan)  # NaN weight -> 1 (NormalizationKernels.metal:75-77)
    wr[99] = np.float16(np.inf)
    g["rms_x"], g["rms_w"] = xr, wr
    g["rms_shape"] = np.array([rr, nn], dtype=np.int64)
    g["rms_eps"] = np.array([1e-5], dtype=np.float32)
    g["rms_y"] = O.ref_rmsnorm_f16(xr, wr, rr, nn, 1e-5)

    # --- RoPE (kernel_rope_f16_inplace), theta 500000 --------------------------
    seq, heads = 3, 8
    data = O.gen_f16(seed=9, stream=1, n=seq * heads * 128)
    g["rope_in"] = data
    g["rope_shape"] = np.array([seq, heads, 128], dtype=np.int64)
    for pos in (0, 2047):
        a = O.rope_args(pos_offset=pos)
        g[f"rope_out_pos{pos}"] = O.ref_rope_f16(a, data, seq, heads)
    # YaRN blend and frequency factors
    ff = (1.0 + np.arange(64, dtype=np.float32) / 16.0).astype(np.float32)
    ay = O.rope_args(pos_offset=1000, ext_factor=1.0, freq_scale=0.25, n_ctx_orig=8192,
                     has_freq_factors=True)
    g["rope_freqs"] = ff
    g["rope_out_yarn"] = O.ref_rope_f16(ay, data, seq, heads, ff)

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
