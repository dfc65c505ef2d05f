"""ctypes/numpy front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Only the tests, ``__graft_entry__.smoke()`` and the bench's CPU-baseline leg
import this module, as the checker.  The product (``metallm_b200``) never
does.

Two libraries sit behind it:

* ``liboracle.so`` -- the C restatement (``q4k_oracle.c``) of the
  reference's Q4_K / RMSNorm / RoPE / attention arithmetic, plus the seeded
  generators shared bit-for-bit with the CUDA generators.
* ``_ref/libmetal_ref.so`` -- the reference's own Metal kernels
  (``MetalLM/Backend/Metal/*.metal``) compiled as host C++; present when the
  reference checkout was available at build time.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_lib: Optional[ctypes.CDLL] = None
_ref: Optional[ctypes.CDLL] = None

QK_K = 256
BLOCK_BYTES = 144
Q6K_BLOCK_BYTES = 210

c_u64 = ctypes.c_uint64
c_vp = ctypes.c_void_p


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError(f"oracle library missing: {path} (run `make -C oracle`)")
        L = ctypes.CDLL(path)
        L.orc_rng_u64.restype = c_u64
        L.orc_rng_u64.argtypes = [c_u64, c_u64, c_u64]
        L.orc_normal.restype = ctypes.c_double
        L.orc_normal.argtypes = [c_u64, c_u64, c_u64]
        L.orc_gen_q4k.argtypes = [c_u64, c_u64, c_u64, c_u64, c_vp]
        L.orc_gen_f16.argtypes = [c_u64, c_u64, c_u64, c_u64, ctypes.c_float, ctypes.c_float, c_vp]
        L.orc_gen_f32.argtypes = [c_u64, c_u64, c_u64, c_u64, ctypes.c_float, ctypes.c_float, c_vp]
        L.orc_q4k_dequant_f32.argtypes = [c_vp, c_u64, c_vp, ctypes.c_int]
        L.orc_q4k_dequant_f16.argtypes = [c_vp, c_u64, c_vp, ctypes.c_int]
        L.orc_q4k_matvec.argtypes = [c_vp, ctypes.c_int, ctypes.c_int, c_vp, c_vp, ctypes.c_int, ctypes.c_int]
        L.orc_q4k_matvec_f32x.argtypes = [c_vp, ctypes.c_int, ctypes.c_int, c_vp, c_vp, ctypes.c_int]
        L.orc_rmsnorm_f16.argtypes = [c_vp, c_vp, c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_rmsnorm_f32.argtypes = [c_vp, c_vp, c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_rope_f16.argtypes = [c_vp, c_vp, c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_rope_f32.argtypes = [c_vp, c_vp, c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_attn_decode.argtypes = [c_vp, c_vp, c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, c_vp, ctypes.c_int]
        L.orc_silu_mul.argtypes = [c_vp, c_vp, c_vp, ctypes.c_int]
        L.orc_q4k_dequant_canonical_f32.argtypes = [c_vp, c_u64, c_vp]
        L.orc_q4k_canonical_to_interleaved.argtypes = [c_vp, c_vp, c_u64]
        L.orc_gen_q6k.argtypes = [c_u64, c_u64, c_u64, c_u64, c_vp]
        L.orc_q6k_dequant_f32.argtypes = [c_vp, c_u64, c_vp, ctypes.c_int]
        L.orc_q6k_matvec.argtypes = [c_vp, ctypes.c_int, ctypes.c_int, c_vp, c_vp, ctypes.c_int]
        _lib = L
    return _lib


def ref_lib() -> Optional[ctypes.CDLL]:
    """The reference's Metal kernels compiled for the host, or None."""
    global _ref
    if _ref is None:
        path = os.path.join(_HERE, "_ref", "libmetal_ref.so")
        if not os.path.exists(path):
            return None
        R = ctypes.CDLL(path)
        R.ref_q4k_dequant_f32.argtypes = [c_vp, c_vp, c_u64, ctypes.c_int]
        R.ref_q4k_dequant_f16.argtypes = [c_vp, c_vp, c_u64, ctypes.c_int]
        R.ref_q4k_matvec.argtypes = [c_vp, ctypes.c_int, ctypes.c_int, c_vp, c_vp, ctypes.c_int]
        R.ref_rmsnorm_f16.argtypes = [c_vp, c_vp, c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        R.ref_rope_f16.argtypes = [c_vp, c_vp, ctypes.c_uint32, ctypes.c_float, ctypes.c_float,
                                   ctypes.c_int32, ctypes.c_int32, ctypes.c_float, ctypes.c_float,
                                   ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int]
        R.ref_silu_f16.argtypes = [c_vp, c_vp, c_u64]
        R.ref_mul_f16.argtypes = [c_vp, c_vp, c_vp, c_u64]
        R.ref_repeat_kv_f16.argtypes = [c_vp, c_vp, ctypes.c_uint32, ctypes.c_uint32,
                                        ctypes.c_uint32, ctypes.c_uint32]
        R.ref_threads_available.restype = ctypes.c_int
        R.ref_q6k_dequant_f32.argtypes = [c_vp, c_vp, c_u64, ctypes.c_int]
        _ref = R
    return _ref


# ----------------------------------------------------------------------------
# generators (bit-identical to metallm_b200's device generators)
# ----------------------------------------------------------------------------

def gen_q4k(seed: int, stream: int, nblocks: int, first_block: int = 0) -> np.ndarray:
    out = np.empty(nblocks * BLOCK_BYTES, dtype=np.uint8)
    lib().orc_gen_q4k(seed, stream, first_block, nblocks, _p(out))
    return out


def gen_q6k(seed: int, stream: int, nblocks: int, first_block: int = 0) -> np.ndarray:
    out = np.empty(nblocks * Q6K_BLOCK_BYTES, dtype=np.uint8)
    lib().orc_gen_q6k(seed, stream, first_block, nblocks, _p(out))
    return out


def gen_f16(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0,
            first: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float16)
    lib().orc_gen_f16(seed, stream, first, n, mean, std, _p(out))
    return out


def gen_f32(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0,
            first: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_gen_f32(seed, stream, first, n, mean, std, _p(out))
    return out


# ----------------------------------------------------------------------------
# restated ops
# ----------------------------------------------------------------------------

def q4k_dequant_f32(blocks: np.ndarray, n: int, nthreads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_q4k_dequant_f32(_p(blocks), n, _p(out), nthreads)
    return out


def q4k_dequant_canonical_f32(blocks: np.ndarray, n: int) -> np.ndarray:
    """Dequant of Q4_K blocks in the GGUF element order (q4k_oracle.h)."""
    out = np.empty(n, dtype=np.float32)
    lib().orc_q4k_dequant_canonical_f32(_p(blocks), n, _p(out))
    return out


def q4k_canonical_to_interleaved(blocks: np.ndarray) -> np.ndarray:
    out = np.empty_like(blocks)
    lib().orc_q4k_canonical_to_interleaved(_p(blocks), _p(out), blocks.size // BLOCK_BYTES)
    return out


def q6k_dequant_f32(blocks: np.ndarray, n: int, nthreads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().orc_q6k_dequant_f32(_p(blocks), n, _p(out), nthreads)
    return out


def q6k_matvec(W: np.ndarray, rows: int, cols: int, x_f16: np.ndarray,
               nthreads: int = 0) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    x = np.ascontiguousarray(x_f16, dtype=np.float16)
    lib().orc_q6k_matvec(_p(W), rows, cols, _p(x), _p(y), nthreads)
    return y


def q4k_dequant_f16(blocks: np.ndarray, n: int, nthreads: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float16)
    lib().orc_q4k_dequant_f16(_p(blocks), n, _p(out), nthreads)
    return out


def q4k_matvec(W: np.ndarray, rows: int, cols: int, x_f16: np.ndarray,
               acc64: bool = True, nthreads: int = 0) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    x = np.ascontiguousarray(x_f16, dtype=np.float16)
    lib().orc_q4k_matvec(_p(W), rows, cols, _p(x), _p(y), int(acc64), nthreads)
    return y


def q4k_matvec_f32x(W: np.ndarray, rows: int, cols: int, x: np.ndarray,
                    nthreads: int = 0) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    lib().orc_q4k_matvec_f32x(_p(W), rows, cols, _p(x), _p(y), nthreads)
    return y


def rmsnorm_f16(x: np.ndarray, w: np.ndarray, rows: int, n: int, eps: float) -> np.ndarray:
    y = np.empty(rows * n, dtype=np.float16)
    x = np.ascontiguousarray(x, dtype=np.float16)
    w = np.ascontiguousarray(w, dtype=np.float16)
    lib().orc_rmsnorm_f16(_p(x), _p(w), _p(y), rows, n, eps)
    return y


def rmsnorm_f32(x: np.ndarray, w: np.ndarray, rows: int, n: int, eps: float) -> np.ndarray:
    y = np.empty(rows * n, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    lib().orc_rmsnorm_f32(_p(x), _p(w), _p(y), rows, n, eps)
    return y


class RopeArgs(ctypes.Structure):
    _fields_ = [("n_dims", ctypes.c_uint32), ("freq_base", ctypes.c_float),
                ("freq_scale", ctypes.c_float), ("pos_offset", ctypes.c_int32),
                ("n_ctx_orig", ctypes.c_int32), ("ext_factor", ctypes.c_float),
                ("attn_factor", ctypes.c_float), ("beta_fast", ctypes.c_float),
                ("beta_slow", ctypes.c_float), ("has_freq_factors", ctypes.c_int32)]


def rope_args(n_dims=128, freq_base=500000.0, freq_scale=1.0, pos_offset=0,
              n_ctx_orig=8192, ext_factor=0.0, attn_factor=1.0, beta_fast=32.0,
              beta_slow=1.0, has_freq_factors=False) -> RopeArgs:
    return RopeArgs(n_dims, freq_base, freq_scale, pos_offset, n_ctx_orig, ext_factor,
                    attn_factor, beta_fast, beta_slow, int(has_freq_factors))


def rope_f16(args: RopeArgs, data: np.ndarray, seq_len: int, num_heads: int,
             head_dim: int, freqs: Optional[np.ndarray] = None) -> np.ndarray:
    d = np.ascontiguousarray(data, dtype=np.float16).copy()
    fp = _p(np.ascontiguousarray(freqs, dtype=np.float32)) if freqs is not None else None
    lib().orc_rope_f16(ctypes.byref(args), _p(d), fp, seq_len, num_heads, head_dim)
    return d


def rope_f32(args: RopeArgs, data: np.ndarray, seq_len: int, num_heads: int,
             head_dim: int, freqs: Optional[np.ndarray] = None) -> np.ndarray:
    d = np.ascontiguousarray(data, dtype=np.float32).copy()
    f = np.ascontiguousarray(freqs, dtype=np.float32) if freqs is not None else None
    lib().orc_rope_f32(ctypes.byref(args), _p(d), _p(f) if f is not None else None,
                       seq_len, num_heads, head_dim)
    return d


def attn_decode(q: np.ndarray, kcache: np.ndarray, vcache: np.ndarray, n_heads: int,
                n_kv: int, head_dim: int, seq_len: int, nthreads: int = 0) -> np.ndarray:
    out = np.empty(n_heads * head_dim, dtype=np.float32)
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(kcache, dtype=np.float16)
    v = np.ascontiguousarray(vcache, dtype=np.float16)
    lib().orc_attn_decode(_p(q), _p(k), _p(v), n_heads, n_kv, head_dim, seq_len, _p(out),
                          nthreads)
    return out


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    out = np.empty_like(g, dtype=np.float32)
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    lib().orc_silu_mul(_p(g), _p(u), _p(out), g.size)
    return out


# ----------------------------------------------------------------------------
# the reference's own kernels, run on the CPU
# ----------------------------------------------------------------------------

def ref_q4k_dequant_f32(blocks: np.ndarray, n: int, nthreads: int = 1) -> np.ndarray:
    R = ref_lib()
    out = np.empty(n, dtype=np.float32)
    R.ref_q4k_dequant_f32(_p(blocks), _p(out), n, nthreads)
    return out


def ref_q6k_dequant_f32(blocks: np.ndarray, n: int, nthreads: int = 1) -> np.ndarray:
    R = ref_lib()
    out = np.empty(n, dtype=np.float32)
    R.ref_q6k_dequant_f32(_p(blocks), _p(out), n, nthreads)
    return out


def ref_q4k_dequant_f16(blocks: np.ndarray, n: int, nthreads: int = 1) -> np.ndarray:
    R = ref_lib()
    out = np.empty(n, dtype=np.float16)
    R.ref_q4k_dequant_f16(_p(blocks), _p(out), n, nthreads)
    return out


def ref_q4k_matvec(W: np.ndarray, rows: int, cols: int, x_f16: np.ndarray,
                   nthreads: int = 1) -> np.ndarray:
    R = ref_lib()
    y = np.empty(rows, dtype=np.float32)
    x = np.ascontiguousarray(x_f16, dtype=np.float16)
    R.ref_q4k_matvec(_p(W), rows, cols, _p(x), _p(y), nthreads)
    return y


def ref_rmsnorm_f16(x: np.ndarray, w: np.ndarray, rows: int, n: int, eps: float) -> np.ndarray:
    R = ref_lib()
    y = np.empty(rows * n, dtype=np.float16)
    x = np.ascontiguousarray(x, dtype=np.float16)
    w = np.ascontiguousarray(w, dtype=np.float16)
    R.ref_rmsnorm_f16(_p(x), _p(w), _p(y), rows, n, eps)
    return y


def ref_rope_f16(args: RopeArgs, data: np.ndarray, seq_len: int, num_heads: int,
                 freqs: Optional[np.ndarray] = None) -> np.ndarray:
    R = ref_lib()
    d = np.ascontiguousarray(data, dtype=np.float16).copy()
    f = np.ascontiguousarray(freqs, dtype=np.float32) if freqs is not None else None
    R.ref_rope_f16(_p(d), _p(f) if f is not None else None, args.n_dims, args.freq_base,
                   args.freq_scale, args.pos_offset, args.n_ctx_orig, args.ext_factor,
                   args.attn_factor, args.beta_fast, args.beta_slow, args.has_freq_factors,
                   seq_len, num_heads)
    return d


def ref_silu_f16(x: np.ndarray) -> np.ndarray:
    R = ref_lib()
    x = np.ascontiguousarray(x, dtype=np.float16)
    y = np.empty_like(x)
    R.ref_silu_f16(_p(x), _p(y), x.size)
    return y


def ref_mul_f16(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    R = ref_lib()
    a = np.ascontiguousarray(a, dtype=np.float16)
    b = np.ascontiguousarray(b, dtype=np.float16)
    y = np.empty_like(a)
    R.ref_mul_f16(_p(a), _p(b), _p(y), a.size)
    return y


def ref_threads() -> int:
    R = ref_lib()
    return int(R.ref_threads_available()) if R is not None else 0
