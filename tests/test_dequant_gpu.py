"""GPU parity of the Q4_K dequantizer and the generators, through the C ABI.

Bar: bit-exact against the reference's kernels (golden vectors) and the
oracle for fp32 and fp16; bf16 equals round-to-nearest-even of the exact
fp32 value.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _bf16_rne(f32: np.ndarray) -> np.ndarray:
    u = f32.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f32)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def test_device_generators_match_oracle(ctx):
    nb = 1000
    buf = ctx.alloc(nb * 144)
    ctx.gen_q4k(42, 9, nb, buf, first_block=123)
    assert np.array_equal(buf.download(np.uint8), O.gen_q4k(42, 9, nb, first_block=123))
    h = ctx.alloc(2 * 5000)
    ctx.gen_f16(7, 3, 5000, h, mean=1.0, std=0.02)
    assert np.array_equal(h.download(np.uint16), O.gen_f16(7, 3, 5000, 1.0, 0.02).view(np.uint16))
    f = ctx.alloc(4 * 5000)
    ctx.gen_f32(7, 4, 5000, f, mean=0.0, std=1.0, first=11)
    assert np.array_equal(f.download(np.uint32), O.gen_f32(7, 4, 5000, first=11).view(np.uint32))


def test_dequant_f32_golden_bitexact(ctx, golden):
    blocks = golden["q4k_blocks"]
    n = golden["q4k_f32"].size
    dB = ctx.to_device(blocks)
    out = ctx.alloc(4 * n)
    ctx.q4k_dequant_f32(dB, out, n)
    got = out.download(np.uint32)
    assert np.array_equal(got, golden["q4k_f32"].view(np.uint32))


def test_dequant_f16_golden_bitexact(ctx, golden):
    blocks = golden["q4k_blocks"]
    n = golden["q4k_f16"].size
    dB = ctx.to_device(blocks)
    out = ctx.alloc(2 * n)
    ctx.q4k_dequant_f16(dB, out, n)
    assert np.array_equal(out.download(np.uint16), golden["q4k_f16"].view(np.uint16))


def test_dequant_ragged_count(ctx, golden):
    n = int(golden["q4k_ragged_n"][0])
    dB = ctx.to_device(golden["q4k_blocks"])
    out = ctx.alloc(4 * golden["q4k_f32"].size)
    ctx.call("mlm_memset", out, 0x7F, out.nbytes)
    ctx.q4k_dequant_f32(dB, out, n)
    got = out.download(np.uint32)
    assert np.array_equal(got[:n], golden["q4k_ragged_f32"].view(np.uint32))
    assert np.all(got[n:] == 0x7F7F7F7F)  # nothing written past n


def test_dequant_config0_full_bitexact(ctx):
    """4096 x 4096 weight: 65,536 blocks -> 16,777,216 fp32 values."""
    nb = 65536
    n = nb * 256
    dB = ctx.alloc(nb * 144)
    ctx.gen_q4k(1234, 0, nb, dB)
    out = ctx.alloc(4 * n)
    ctx.q4k_dequant_f32(dB, out, n)
    ref = O.q4k_dequant_f32(O.gen_q4k(1234, 0, nb), n)
    assert np.array_equal(out.download(np.uint32), ref.view(np.uint32))
    out16 = ctx.alloc(2 * n)
    ctx.q4k_dequant_f16(dB, out16, n)
    ref16 = O.q4k_dequant_f16(O.gen_q4k(1234, 0, nb), n)
    assert np.array_equal(out16.download(np.uint16), ref16.view(np.uint16))


def test_dequant_bf16_is_rne_of_exact(ctx, golden):
    blocks = golden["q4k_blocks"]
    n = golden["q4k_f32"].size
    dB = ctx.to_device(blocks)
    out = ctx.alloc(2 * n)
    ctx.q4k_dequant_bf16(dB, out, n)
    assert np.array_equal(out.download(np.uint16), _bf16_rne(golden["q4k_f32"]))


def test_dequant_sync_helper_allocates_and_waits(ctx, golden):
    import ctypes
    blocks = golden["q4k_blocks"]
    n = golden["q4k_f32"].size
    dB = ctx.to_device(blocks)
    p = ctypes.c_void_p()
    ctx.call("mlm_dequantize_q4k_to_f32", dB, n, ctypes.byref(p))
    got = np.empty(n, dtype=np.float32)
    ctx._check(ctx.lib.mlm_download(ctx.handle, got.ctypes.data, p, got.nbytes), "download")
    ctx.lib.mlm_free(ctx.handle, p)
    assert np.array_equal(got.view(np.uint32), golden["q4k_f32"].view(np.uint32))


def test_dequant_rejects_misaligned(ctx, golden):
    from metallm_b200 import MLMError
    dB = ctx.to_device(golden["q4k_blocks"])
    out = ctx.alloc(4 * 512)
    with pytest.raises(MLMError) as e:
        ctx.q4k_dequant_f32(dB.ptr + 4, out, 256)
    assert e.value.status == -3


def test_dequant_zero_elements_is_a_noop(ctx):
    ctx.q4k_dequant_f32(0, 0, 0)
