"""ctypes binding of libmetallm_cuda.so (the C ABI in include/metallm_cuda.h).

The shared library is the product; this module only declares its symbols.
There is no fallback: if the library is missing or no B200 is visible the
calls raise.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libmetallm_cuda.so")

c_int, c_u64, c_vp, c_float, c_size = (ctypes.c_int, ctypes.c_uint64, ctypes.c_void_p,
                                       ctypes.c_float, ctypes.c_size_t)
c_i32p = ctypes.POINTER(ctypes.c_int32)

MLM_OK = 0
STATUS_NAMES = {0: "MLM_OK", -1: "MLM_ERR_ARG", -2: "MLM_ERR_SHAPE", -3: "MLM_ERR_ALIGN",
                -4: "MLM_ERR_ALLOC", -5: "MLM_ERR_CUDA", -6: "MLM_ERR_NCCL",
                -7: "MLM_ERR_TIMEOUT", -8: "MLM_ERR_STATE", -9: "MLM_ERR_UNSUPPORTED"}


class RopeArgs(ctypes.Structure):
    """mlm_rope_args (MetalRopeArgs, PositionalEmbeddingsKernels.metal:15-42)."""
    _fields_ = [("n_dims", ctypes.c_uint32), ("freq_base", c_float), ("freq_scale", c_float),
                ("pos_offset", ctypes.c_int32), ("n_ctx_orig", ctypes.c_int32),
                ("ext_factor", c_float), ("attn_factor", c_float), ("beta_fast", c_float),
                ("beta_slow", c_float), ("has_freq_factors", ctypes.c_int32)]


def rope_args(n_dims=128, freq_base=500000.0, freq_scale=1.0, pos_offset=0, n_ctx_orig=8192,
              ext_factor=0.0, attn_factor=1.0, beta_fast=32.0, beta_slow=1.0,
              has_freq_factors=False) -> RopeArgs:
    return RopeArgs(n_dims, freq_base, freq_scale, pos_offset, n_ctx_orig, ext_factor,
                    attn_factor, beta_fast, beta_slow, int(has_freq_factors))


class LlamaConfig(ctypes.Structure):
    """mlm_llama_config (LlamaConfig as LlamaRunner.swift reads it)."""
    _fields_ = [("n_layers", ctypes.c_int32), ("dim", ctypes.c_int32), ("n_heads", ctypes.c_int32),
                ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("ffn_dim", ctypes.c_int32), ("vocab", ctypes.c_int32), ("max_seq", ctypes.c_int32),
                ("rms_eps", c_float), ("rope", RopeArgs)]


class LlamaLayer(ctypes.Structure):
    """mlm_llama_layer: device pointers of one layer's tensors and the types
    of attn_v and ffn_down."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("attn_norm", "wq", "wk", "wv", "wo", "ffn_norm",
                                               "w_gate", "w_up", "w_down", "k_cache", "v_cache")]
    _fields_ += [("wv_type", ctypes.c_int32), ("w_down_type", ctypes.c_int32)]


class LlamaGlobals(ctypes.Structure):
    """mlm_llama_globals."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("tok_embd", "output_norm", "output", "rope_freqs")]
    _fields_ += [("output_type", ctypes.c_int32)]


TYPE_Q4_K, TYPE_Q6_K = 12, 14  # MLM_TYPE_*: the ggml_type values


class LlamaTypes(ctypes.Structure):
    """mlm_llama_types: the output head's type and per-layer attn_v /
    ffn_down types (NULL arrays: all Q4_K)."""
    _fields_ = [("output", ctypes.c_int32), ("attn_v", ctypes.POINTER(ctypes.c_int32)),
                ("ffn_down", ctypes.POINTER(ctypes.c_int32))]


# (name, restype, argtypes) of every exported entry point
SIGNATURES = [
    ("mlm_abi_version", c_int, []),
    ("mlm_status_string", ctypes.c_char_p, [c_int]),
    ("mlm_create", c_int, [c_int, ctypes.POINTER(c_vp)]),
    ("mlm_destroy", None, [c_vp]),
    ("mlm_last_error", ctypes.c_char_p, [c_vp]),
    ("mlm_device_sm_count", c_int, [c_vp]),
    ("mlm_get_stream", c_int, [c_vp, ctypes.POINTER(c_vp)]),
    ("mlm_set_stream", c_int, [c_vp, c_vp]),
    ("mlm_alloc", c_int, [c_vp, c_size, ctypes.POINTER(c_vp)]),
    ("mlm_free", c_int, [c_vp, c_vp]),
    ("mlm_memset", c_int, [c_vp, c_vp, c_int, c_size]),
    ("mlm_upload", c_int, [c_vp, c_vp, c_vp, c_size]),
    ("mlm_download", c_int, [c_vp, c_vp, c_vp, c_size]),
    ("mlm_upload_async", c_int, [c_vp, c_vp, c_vp, c_size]),
    ("mlm_download_async", c_int, [c_vp, c_vp, c_vp, c_size]),
    ("mlm_host_alloc", c_int, [c_vp, c_size, ctypes.POINTER(c_vp)]),
    ("mlm_host_free", c_int, [c_vp, c_vp]),
    ("mlm_commit", c_int, [c_vp]),
    ("mlm_graph_begin", c_int, [c_vp]),
    ("mlm_graph_end", c_int, [c_vp, ctypes.POINTER(c_vp)]),
    ("mlm_graph_launch", c_int, [c_vp, c_vp]),
    ("mlm_graph_destroy", None, [c_vp]),
    ("mlm_wait", c_int, [c_vp]),
    ("mlm_gen_q4k", c_int, [c_vp, c_u64, c_u64, c_u64, c_u64, c_vp]),
    ("mlm_gen_q4k_sub", c_int, [c_vp, c_u64, c_u64, c_u64, c_u64, c_u64, c_u64, c_u64, c_vp]),
    ("mlm_gen_f16", c_int, [c_vp, c_u64, c_u64, c_u64, c_u64, c_float, c_float, c_vp]),
    ("mlm_gen_f32", c_int, [c_vp, c_u64, c_u64, c_u64, c_u64, c_float, c_float, c_vp]),
    ("mlm_q4k_dequant_f32", c_int, [c_vp, c_vp, c_vp, c_u64]),
    ("mlm_q4k_dequant_f16", c_int, [c_vp, c_vp, c_vp, c_u64]),
    ("mlm_q4k_dequant_bf16", c_int, [c_vp, c_vp, c_vp, c_u64]),
    ("mlm_q4k_repack_canonical", c_int, [c_vp, c_vp, c_vp, c_u64]),
    ("mlm_gen_q6k", c_int, [c_vp, c_u64, c_u64, c_u64, c_u64, c_vp]),
    ("mlm_gen_q6k_sub", c_int, [c_vp, c_u64, c_u64, c_u64, c_u64, c_u64, c_u64, c_u64, c_vp]),
    ("mlm_q6k_dequant_f32", c_int, [c_vp, c_vp, c_vp, c_u64]),
    ("mlm_q6k_dequant_f16", c_int, [c_vp, c_vp, c_vp, c_u64]),
    ("mlm_q6k_dequant_bf16", c_int, [c_vp, c_vp, c_vp, c_u64]),
    ("mlm_q6k_gemv", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    ("mlm_q6k_gemv_xs", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp]),
    ("mlm_q6k_gemv_rmsnorm", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_vp]),
    ("mlm_q6k_gemv_swiglu", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp]),
    ("mlm_q6k_gemm", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_int, c_vp, c_vp, c_vp]),
    ("mlm_dequantize_q4k_to_f32", c_int, [c_vp, c_vp, c_u64, ctypes.POINTER(c_vp)]),
    ("mlm_dequantize_q4k_to_f16", c_int, [c_vp, c_vp, c_u64, ctypes.POINTER(c_vp)]),
    ("mlm_q4k_gemv", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    ("mlm_q4k_gemv_xs", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp]),
    ("mlm_q4k_gemv_rmsnorm", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_vp]),
    ("mlm_q4k_gemv_swiglu", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp, c_vp]),
    ("mlm_q4k_gemv_gate_up", c_int,
     [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_float, c_vp, c_vp, c_vp]),
    ("mlm_q4k_gemm", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_int, c_vp, c_vp]),
    ("mlm_q4k_gemv_batch", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_int, c_vp, c_vp]),
    ("mlm_q4k_gemv_static", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp, c_vp]),
    ("mlm_q4k_gemv_plan", c_int, [c_int, c_int, c_int, c_i32p, c_i32p, c_i32p]),
    ("mlm_q4k_gemv_batch_plan", c_int, [c_int, c_int, c_int, c_i32p, c_i32p]),
    ("mlm_rmsnorm_f16", c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_float]),
    ("mlm_rmsnorm_f32", c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_float]),
    ("mlm_rope_f16", c_int, [c_vp, c_vp, c_vp, ctypes.POINTER(RopeArgs), c_int, c_int, c_int]),
    ("mlm_rope_qk_kv_append", c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, ctypes.POINTER(RopeArgs),
                                      c_int, c_int, c_int, c_vp, c_vp, c_vp, c_int]),
    ("mlm_silu_mul", c_int, [c_vp, c_vp, c_vp, c_vp, c_int]),
    ("mlm_silu_mul_scaled", c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_int]),
    ("mlm_add_f32", c_int, [c_vp, c_vp, c_vp, c_vp, c_int]),
    ("mlm_attn_decode", c_int, [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp]),
    ("mlm_embed_f16", c_int, [c_vp, c_vp, c_int, c_int, c_vp, c_vp]),
    ("mlm_argmax_f32", c_int, [c_vp, c_vp, c_int, c_vp]),
    ("mlm_llama_create", c_int, [c_vp, ctypes.POINTER(LlamaConfig), ctypes.POINTER(c_vp)]),
    ("mlm_llama_destroy", None, [c_vp]),
    ("mlm_llama_layer_tensors", c_int, [c_vp, c_int, ctypes.POINTER(LlamaLayer)]),
    ("mlm_llama_global_tensors", c_int, [c_vp, ctypes.POINTER(LlamaGlobals)]),
    ("mlm_llama_reset", c_int, [c_vp]),
    ("mlm_llama_set_position", c_int, [c_vp, c_int]),
    ("mlm_llama_position", c_int, [c_vp]),
    ("mlm_llama_forward_layer", c_int, [c_vp, c_int, c_vp]),
    ("mlm_llama_forward", c_int, [c_vp, c_int, c_vp]),
    ("mlm_llama_prefill", c_int, [c_vp, ctypes.POINTER(ctypes.c_int32), c_int, c_vp, c_vp]),
    ("mlm_llama_decode_greedy", c_int, [c_vp, c_int, c_int, c_vp]),
    ("mlm_llama_create_batch", c_int, [c_vp, c_vp, c_int, ctypes.POINTER(c_vp)]),
    ("mlm_llama_create_typed", c_int, [c_vp, c_vp, c_int, c_vp, ctypes.POINTER(c_vp)]),
    ("mlm_llama_prefill_seq", c_int, [c_vp, c_int, c_vp, c_int, c_vp, c_vp]),
    ("mlm_llama_seq_position", c_int, [c_vp, c_int]),
    ("mlm_llama_forward_batch", c_int, [c_vp, c_vp, c_vp]),
    ("mlm_llama_decode_greedy_batch", c_int, [c_vp, c_vp, c_int, c_vp]),
    ("mlm_tp_unique_id", c_int, [c_vp, c_vp, c_size]),
    ("mlm_tp_init", c_int, [c_vp, c_int, c_int, c_vp]),
    ("mlm_tp_info", c_int, [c_vp, ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    ("mlm_tp_allreduce_f32", c_int, [c_vp, c_vp, c_vp, c_size]),
    ("mlm_tp_allgather", c_int, [c_vp, c_vp, c_vp, c_size]),
]

_lib: Optional[ctypes.CDLL] = None


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the CUDA library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError(
            f"libmetallm_cuda.so not found at {path}; build it with "
            "`python -m metallm_b200.build` (there is no CPU fallback)")
    lib = ctypes.CDLL(path)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class MLMError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
