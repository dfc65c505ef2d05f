"""metallm_b200 -- B200 (sm_100a) implementation of MetalLM's Q4_K Llama-3 hot path.

The product is the C-ABI shared library ``libmetallm_cuda.so`` (declared in
``include/metallm_cuda.h``).  This package holds its CUDA sources
(``csrc/``), the in-tree build (``build.py``) and a thin Python binding
(``Context``/``DeviceBuffer``) used by the tests and the bench.  Every call
goes through the C ABI; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import weakref
from typing import Optional, Sequence

import numpy as np

from ._lib import (LIB_PATH, TYPE_Q4_K, TYPE_Q6_K, LlamaConfig, LlamaGlobals,  # noqa: F401
                   LlamaLayer, LlamaTypes, MLMError, RopeArgs, load, rope_args)

QK_K = 256
Q4K_BLOCK_BYTES = 144


class DeviceBuffer:
    """A device allocation made through mlm_alloc (freed with mlm_free)."""

    def __init__(self, ctx: "Context", nbytes: int):
        self.ctx = ctx
        self.nbytes = int(nbytes)
        p = ctypes.c_void_p()
        ctx._check(ctx.lib.mlm_alloc(ctx.handle, self.nbytes, ctypes.byref(p)), "mlm_alloc")
        self.ptr = int(p.value)

    def free(self) -> None:
        if self.ptr:
            self.ctx.lib.mlm_free(self.ctx.handle, ctypes.c_void_p(self.ptr))
            self.ptr = 0

    def __del__(self):
        try:
            if self.ptr and self.ctx.handle:
                self.free()
        except Exception:
            pass

    def upload(self, a: np.ndarray) -> "DeviceBuffer":
        a = np.ascontiguousarray(a)
        assert a.nbytes <= self.nbytes, (a.nbytes, self.nbytes)
        self.ctx._check(self.ctx.lib.mlm_upload(self.ctx.handle, ctypes.c_void_p(self.ptr),
                                                a.ctypes.data, a.nbytes), "mlm_upload")
        return self

    def download(self, dtype, count: Optional[int] = None) -> np.ndarray:
        dtype = np.dtype(dtype)
        n = self.nbytes // dtype.itemsize if count is None else int(count)
        out = np.empty(n, dtype=dtype)
        self.ctx._check(self.ctx.lib.mlm_download(self.ctx.handle, out.ctypes.data,
                                                  ctypes.c_void_p(self.ptr), out.nbytes),
                        "mlm_download")
        return out

    def __int__(self) -> int:
        return self.ptr


class Context:
    """One mlm_ctx: a device, a stream and the kernels' scratch."""

    def __init__(self, device: int = 0):
        self.lib = load()
        h = ctypes.c_void_p()
        st = self.lib.mlm_create(device, ctypes.byref(h))
        if st != 0:
            raise MLMError(st, f"mlm_create(device={device}) failed "
                               f"({self.lib.mlm_status_string(st).decode()})")
        self.handle = h
        self.device = device
        # runners made on this context; closed before the context itself so
        # that no runner outlives the stream and scratch it uses
        self._runners = weakref.WeakSet()

    def close(self) -> None:
        if self.handle:
            for r in list(self._runners):
                r.close()
            self.lib.mlm_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- plumbing ------------------------------------------------------------
    def _check(self, status: int, what: str) -> None:
        if status != 0:
            msg = self.lib.mlm_last_error(self.handle)
            raise MLMError(status, f"{what}: {msg.decode() if msg else ''}")

    def call(self, name: str, *args) -> None:
        fn = getattr(self.lib, name)
        conv = [ctypes.c_void_p(int(a)) if isinstance(a, DeviceBuffer) else a for a in args]
        self._check(fn(self.handle, *conv), name)

    def alloc(self, nbytes: int) -> DeviceBuffer:
        return DeviceBuffer(self, nbytes)

    def to_device(self, a: np.ndarray) -> DeviceBuffer:
        a = np.ascontiguousarray(a)
        return DeviceBuffer(self, max(a.nbytes, 16)).upload(a)

    def wait(self) -> None:
        self._check(self.lib.mlm_wait(self.handle), "mlm_wait")

    def stream(self) -> int:
        s = ctypes.c_void_p()
        self._check(self.lib.mlm_get_stream(self.handle, ctypes.byref(s)), "mlm_get_stream")
        return int(s.value or 0)

    def set_stream(self, stream: int) -> None:
        self._check(self.lib.mlm_set_stream(self.handle, ctypes.c_void_p(stream)),
                    "mlm_set_stream")

    # -- tensor parallelism (one context per rank) ------------------------------
    @staticmethod
    def _nccl_first() -> None:
        """The library binds the NCCL already in the process when there is one.
        PyTorch links its own NCCL build; loading it now, before the library
        would fall back to the system's copy, keeps a single NCCL per process."""
        try:
            import torch.distributed  # noqa: F401
        except ImportError:
            pass

    def tp_unique_id(self) -> bytes:
        self._nccl_first()
        buf = ctypes.create_string_buffer(128)
        self._check(self.lib.mlm_tp_unique_id(self.handle, buf, 128), "mlm_tp_unique_id")
        return buf.raw

    def tp_init(self, nranks: int, rank: int, unique_id: bytes) -> None:
        self._nccl_first()
        buf = ctypes.create_string_buffer(bytes(unique_id), 128)
        self._check(self.lib.mlm_tp_init(self.handle, nranks, rank, buf), "mlm_tp_init")

    def tp_info(self) -> tuple:
        """(rank, size) of this context's group; size 0 without one."""
        r, n = ctypes.c_int(), ctypes.c_int()
        self._check(self.lib.mlm_tp_info(self.handle, ctypes.byref(r), ctypes.byref(n)),
                    "mlm_tp_info")
        return r.value, n.value

    # -- CUDA graphs -----------------------------------------------------------
    def graph_begin(self) -> None:
        self._check(self.lib.mlm_graph_begin(self.handle), "mlm_graph_begin")

    def graph_end(self) -> "Graph":
        g = ctypes.c_void_p()
        self._check(self.lib.mlm_graph_end(self.handle, ctypes.byref(g)), "mlm_graph_end")
        return Graph(self, g)

    @property
    def sm_count(self) -> int:
        return int(self.lib.mlm_device_sm_count(self.handle))

    # -- generators ----------------------------------------------------------
    def gen_q4k(self, seed: int, stream: int, nblocks: int, out: DeviceBuffer,
                first_block: int = 0) -> DeviceBuffer:
        self.call("mlm_gen_q4k", seed, stream, first_block, nblocks, out)
        return out

    def gen_q4k_sub(self, seed: int, stream: int, nb_full: int, row0: int, rows: int, kb0: int,
                    nkb: int, out) -> None:
        """Rows row0.. and block columns kb0.. of generated tensor `stream`."""
        self.call("mlm_gen_q4k_sub", seed, stream, nb_full, row0, rows, kb0, nkb,
                  ctypes.c_void_p(int(out)))

    def gen_q6k_sub(self, seed: int, stream: int, nb_full: int, row0: int, rows: int, kb0: int,
                    nkb: int, out) -> None:
        """The same for a generated Q6_K tensor."""
        self.call("mlm_gen_q6k_sub", seed, stream, nb_full, row0, rows, kb0, nkb,
                  ctypes.c_void_p(int(out)))

    def gen_f16(self, seed: int, stream: int, n: int, out: DeviceBuffer, mean: float = 0.0,
                std: float = 1.0, first: int = 0) -> DeviceBuffer:
        self.call("mlm_gen_f16", seed, stream, first, n, ctypes.c_float(mean),
                  ctypes.c_float(std), out)
        return out

    def gen_f32(self, seed: int, stream: int, n: int, out: DeviceBuffer, mean: float = 0.0,
                std: float = 1.0, first: int = 0) -> DeviceBuffer:
        self.call("mlm_gen_f32", seed, stream, first, n, ctypes.c_float(mean),
                  ctypes.c_float(std), out)
        return out

    # -- ops (thin wrappers; all stream-ordered) ------------------------------
    def q4k_dequant_f32(self, blocks, out, n: int) -> None:
        self.call("mlm_q4k_dequant_f32", blocks, out, n)

    def q4k_dequant_f16(self, blocks, out, n: int) -> None:
        self.call("mlm_q4k_dequant_f16", blocks, out, n)

    def q4k_dequant_bf16(self, blocks, out, n: int) -> None:
        self.call("mlm_q4k_dequant_bf16", blocks, out, n)

    def q4k_gemv(self, W, rows: int, cols: int, x, y, residual=None) -> None:
        self.call("mlm_q4k_gemv", W, rows, cols, x, y, residual)

    def q4k_repack_canonical(self, src, dst, nblocks: int) -> None:
        """GGUF-order Q4_K blocks into the order every op here reads."""
        self.call("mlm_q4k_repack_canonical", src, dst, nblocks)

    def gen_q6k(self, seed: int, stream: int, nblocks: int, out: DeviceBuffer,
                first_block: int = 0) -> DeviceBuffer:
        self.call("mlm_gen_q6k", seed, stream, first_block, nblocks, out)
        return out

    def q6k_dequant_f32(self, blocks, out, n: int) -> None:
        self.call("mlm_q6k_dequant_f32", blocks, out, n)

    def q6k_dequant_f16(self, blocks, out, n: int) -> None:
        self.call("mlm_q6k_dequant_f16", blocks, out, n)

    def q6k_dequant_bf16(self, blocks, out, n: int) -> None:
        self.call("mlm_q6k_dequant_bf16", blocks, out, n)

    def q6k_gemv(self, W, rows: int, cols: int, x, y, residual=None) -> None:
        self.call("mlm_q6k_gemv", W, rows, cols, x, y, residual)


class Graph:
    """A captured op sequence (mlm_graph)."""

    def __init__(self, ctx: Context, handle: ctypes.c_void_p):
        self.ctx = ctx
        self.handle = handle

    def launch(self) -> None:
        self.ctx._check(self.ctx.lib.mlm_graph_launch(self.ctx.handle, self.handle),
                        "mlm_graph_launch")

    def destroy(self) -> None:
        if self.handle:
            self.ctx.lib.mlm_graph_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class Llama:
    """mlm_llama: the decode runner (LlamaRunner.swift) on one context.

    Tensors live in the runner's own device buffers; ``layer_tensors`` and
    ``global_tensors`` give their device addresses (as ints) so a loader can
    write the raw GGUF blocks straight into them.
    """

    def __init__(self, ctx: Context, cfg: LlamaConfig, batch: int = 1,
                 types: Optional[dict] = None):
        """types (a Q4_K_M file's per-tensor types): {"output": TYPE_Q6_K,
        "attn_v": [type per layer], "ffn_down": [type per layer]}; missing
        entries are Q4_K."""
        self.ctx = ctx
        self.cfg = cfg
        self.batch = batch
        h = ctypes.c_void_p()
        if types:
            arr = lambda v: ((ctypes.c_int32 * cfg.n_layers)(*v) if v is not None else None)
            av, fd = arr(types.get("attn_v")), arr(types.get("ffn_down"))
            t = LlamaTypes(int(types.get("output", TYPE_Q4_K)),
                           ctypes.cast(av, ctypes.POINTER(ctypes.c_int32)) if av else None,
                           ctypes.cast(fd, ctypes.POINTER(ctypes.c_int32)) if fd else None)
            st = ctx.lib.mlm_llama_create_typed(ctx.handle, ctypes.byref(cfg), batch,
                                                ctypes.byref(t), ctypes.byref(h))
        elif batch == 1:
            st = ctx.lib.mlm_llama_create(ctx.handle, ctypes.byref(cfg), ctypes.byref(h))
        else:
            st = ctx.lib.mlm_llama_create_batch(ctx.handle, ctypes.byref(cfg), batch,
                                                ctypes.byref(h))
        ctx._check(st, "mlm_llama_create")
        self.handle = h
        ctx._runners.add(self)

    def _check(self, st: int, what: str) -> None:
        self.ctx._check(st, what)

    def layer_tensors(self, layer: int) -> dict:
        t = LlamaLayer()
        self._check(self.ctx.lib.mlm_llama_layer_tensors(self.handle, layer, ctypes.byref(t)),
                    "mlm_llama_layer_tensors")
        return {name: int(getattr(t, name)) for name, _ in LlamaLayer._fields_}

    def global_tensors(self) -> dict:
        t = LlamaGlobals()
        self._check(self.ctx.lib.mlm_llama_global_tensors(self.handle, ctypes.byref(t)),
                    "mlm_llama_global_tensors")
        return {name: int(getattr(t, name)) for name, _ in LlamaGlobals._fields_}

    def reset(self) -> None:
        self._check(self.ctx.lib.mlm_llama_reset(self.handle), "mlm_llama_reset")

    def set_position(self, pos: int) -> None:
        self._check(self.ctx.lib.mlm_llama_set_position(self.handle, pos), "mlm_llama_set_position")

    @property
    def position(self) -> int:
        return int(self.ctx.lib.mlm_llama_position(self.handle))

    def forward_layer(self, layer: int, hidden) -> None:
        self._check(self.ctx.lib.mlm_llama_forward_layer(self.handle, layer,
                                                         ctypes.c_void_p(int(hidden))),
                    "mlm_llama_forward_layer")

    def forward(self, token: int, logits=None) -> None:
        self._check(self.ctx.lib.mlm_llama_forward(
            self.handle, token, ctypes.c_void_p(int(logits)) if logits is not None else None),
            "mlm_llama_forward")

    def prefill(self, tokens: Sequence[int], next_token=None, logits=None, seq: int = 0) -> None:
        arr = (ctypes.c_int32 * len(tokens))(*[int(t) for t in tokens])
        lg = ctypes.c_void_p(int(logits)) if logits is not None else None
        nx = ctypes.c_void_p(int(next_token)) if next_token is not None else None
        if seq == 0:
            st = self.ctx.lib.mlm_llama_prefill(self.handle, arr, len(tokens), lg, nx)
        else:
            st = self.ctx.lib.mlm_llama_prefill_seq(self.handle, seq, arr, len(tokens), lg, nx)
        self._check(st, "mlm_llama_prefill")

    def seq_position(self, seq: int) -> int:
        return int(self.ctx.lib.mlm_llama_seq_position(self.handle, seq))

    def forward_batch(self, tokens: Sequence[int], logits=None) -> None:
        """One step of every sequence; logits fp32 [batch][vocab] on the device."""
        arr = (ctypes.c_int32 * self.batch)(*[int(t) for t in tokens])
        self._check(self.ctx.lib.mlm_llama_forward_batch(
            self.handle, arr, ctypes.c_void_p(int(logits)) if logits is not None else None),
            "mlm_llama_forward_batch")

    def decode_greedy_batch(self, tokens: Sequence[int], steps: int, tokens_out) -> None:
        """`steps` greedy steps of every sequence; tokens_out int32 [steps][batch]."""
        arr = (ctypes.c_int32 * self.batch)(*[int(t) for t in tokens])
        self._check(self.ctx.lib.mlm_llama_decode_greedy_batch(
            self.handle, arr, steps, ctypes.c_void_p(int(tokens_out))),
            "mlm_llama_decode_greedy_batch")

    def decode_greedy(self, token: int, steps: int, tokens_out) -> None:
        self._check(self.ctx.lib.mlm_llama_decode_greedy(self.handle, token, steps,
                                                         ctypes.c_void_p(int(tokens_out))),
                    "mlm_llama_decode_greedy")

    def close(self) -> None:
        if self.handle and self.ctx.handle:
            self.ctx.lib.mlm_llama_destroy(self.handle)
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def exported_symbols() -> Sequence[str]:
    from ._lib import SIGNATURES
    return [s[0] for s in SIGNATURES]
