# SPDX-License-Identifier: Apache-2.0
"""ctypes binding of libkllm_gpu (the B200 paged-attention backend).

The product host code is C (``csrc/kllm_shim.c``); this module only mirrors
the C ABI declared in ``include/kllm_gpu.h`` so Python tests and the
benchmark can call it exactly as a C caller would (``userspace/compute/
infer_gpu.c:167-211`` is the reference caller). There is no Python fallback:
if the shared library is missing, :func:`load` raises.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, Structure, c_float, c_int, c_uint8, c_uint32,
                    c_uint64, c_void_p)

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(ROOT_DIR, "lib", "libkllm_gpu.so")
HEADER_PATH = os.path.join(os.path.dirname(ROOT_DIR), "include", "kllm_gpu.h")

# enum kllm_gpu_backend (userspace/gpu/gpu_attention.h:19-24)
KLLM_GPU_NONE, KLLM_GPU_XE, KLLM_GPU_CUDA, KLLM_GPU_ROCM = 0, 1, 2, 3
# enum kllm_kv_dtype
KV_BF16, KV_MX_FP8, KV_MX_BF16_COMPAT = 0, 1, 2
# error codes
OK, EIO, ENOMEM, ENODEV, EINVAL, ENOSPC, ENOSYS, ETIMEDOUT = 0, -5, -12, -19, -22, -28, -38, -110
ERR_SEQ_TOO_LONG, ERR_MISALIGNED, ERR_APPEND_NOPAGE, ERR_TIMEOUT = 0x1, 0x2, 0x4, 0x8
ERR_TOPK_RANGE, ERR_NONFINITE, ERR_PAGE_RANGE = 0x10, 0x20, 0x40
TRACE_DECODE, TRACE_APPEND, TRACE_PREFILL = 1, 2, 3


class TraceRecord(Structure):
    """struct kllm_gpu_trace_record"""
    _fields_ = [("seq", c_uint64), ("tag", c_uint64), ("submit_ns", c_uint64),
                ("op", c_uint32), ("gpu_us", c_float)]
DECODE_OVERLAP_PREV = 0x1   # kllm_gpu_attention_params_v2.flags


class AttnParams(Structure):
    """struct kllm_gpu_attention_params (userspace/gpu/gpu_attention.h:26-38)."""
    _fields_ = [("output", c_void_p), ("query", c_void_p), ("block_tables", c_void_p),
                ("seq_lens", c_void_p), ("num_seqs", c_int), ("num_heads", c_int),
                ("num_kv_heads", c_int), ("head_dim", c_int),
                ("max_blocks_per_seq", c_int), ("scale", c_float), ("stream", c_void_p)]


class AttnParamsV2(Structure):
    _fields_ = [("struct_size", c_uint32), ("flags", c_uint32), ("output", c_void_p),
                ("query", c_void_p), ("block_tables", c_void_p), ("seq_lens", c_void_p),
                ("num_seqs", c_int), ("num_heads", c_int), ("num_kv_heads", c_int),
                ("head_dim", c_int), ("max_blocks_per_seq", c_int), ("block_size", c_int),
                ("kv_dtype", c_int), ("layer", c_int), ("layer_stride", c_uint64),
                ("scale", c_float), ("split", c_int), ("partial_m", c_void_p),
                ("partial_l", c_void_p), ("partial_o", c_void_p), ("err_word", c_void_p),
                ("workspace", c_void_p), ("workspace_size", c_uint64), ("stream", c_void_p)]


class KvAppendParams(Structure):
    _fields_ = [("struct_size", c_uint32), ("flags", c_uint32), ("k", c_void_p),
                ("v", c_void_p), ("token_seq", c_void_p), ("token_pos", c_void_p),
                ("num_tokens", c_int), ("num_seqs", c_int), ("block_tables", c_void_p),
                ("max_blocks_per_seq", c_int), ("num_kv_heads", c_int), ("head_dim", c_int),
                ("block_size", c_int), ("kv_dtype", c_int), ("layer", c_int),
                ("layer_stride", c_uint64), ("err_word", c_void_p), ("stream", c_void_p)]


class GatherParams(Structure):
    _fields_ = [("struct_size", c_uint32), ("flags", c_uint32), ("k_out", c_void_p),
                ("v_out", c_void_p), ("counts_out", c_void_p), ("block_tables", c_void_p),
                ("seq_lens", c_void_p), ("num_seqs", c_int), ("num_kv_heads", c_int),
                ("head_dim", c_int), ("max_blocks_per_seq", c_int), ("block_size", c_int),
                ("kv_dtype", c_int), ("layer", c_int), ("layer_stride", c_uint64),
                ("stream", c_void_p)]


class PrefillParams(Structure):
    _fields_ = [("struct_size", c_uint32), ("flags", c_uint32), ("output", c_void_p),
                ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("cu_seqlens", c_void_p),
                ("ctx_lens", c_void_p), ("num_seqs", c_int), ("num_tokens", c_int),
                ("max_chunk", c_int), ("num_heads", c_int), ("num_kv_heads", c_int),
                ("head_dim", c_int), ("block_tables", c_void_p), ("max_blocks_per_seq", c_int),
                ("block_size", c_int), ("kv_dtype", c_int), ("layer", c_int),
                ("layer_stride", c_uint64), ("scale", c_float), ("append", c_int),
                ("err_word", c_void_p), ("stream", c_void_p)]


class TableBuildParams(Structure):
    _fields_ = [("struct_size", c_uint32), ("flags", c_uint32), ("token_ids", c_void_p),
                ("token_starts", c_void_p), ("seq_lens", c_void_p), ("first_block", c_void_p),
                ("num_seqs", c_int), ("max_blocks_per_seq", c_int), ("block_size", c_int),
                ("index", c_void_p), ("index_capacity", c_uint32), ("now_ns", c_uint64),
                ("arena_base", c_uint64), ("slot_bytes", c_uint64), ("total_slots", c_uint64),
                ("k_offset", c_uint64), ("v_offset", c_uint64), ("block_tables", c_void_p),
                ("hashes", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_uint64),
                ("miss_list", c_void_p), ("miss_capacity", c_int), ("miss_count", c_void_p),
                ("hit_miss", c_void_p), ("err_word", c_void_p), ("stream", c_void_p)]


class LmHeadParams(Structure):
    _fields_ = [("struct_size", c_uint32), ("flags", c_uint32), ("hidden", c_void_p),
                ("weight", c_void_p), ("num_rows", c_int), ("hidden_dim", c_int), ("vocab", c_int),
                ("logits", c_void_p), ("method", c_void_p), ("temperature", c_void_p),
                ("top_k", c_void_p), ("uniform", c_void_p), ("tokens", c_void_p),
                ("workspace", c_void_p), ("workspace_bytes", c_uint64), ("err_word", c_void_p),
                ("stream", c_void_p)]


SAMPLE_GREEDY, SAMPLE_TOP_K, SAMPLE_TOP_P, SAMPLE_TEMPERATURE = 0, 1, 2, 3


class WfBlockDesc(Structure):
    """userspace/gpu/nvme_ep_wavefront.h:32-39"""
    _fields_ = [("obj_key", c_uint8 * 32), ("vram_dest_addr", c_uint64), ("block_size", c_uint32),
                ("layer_start", c_uint32), ("layer_count", c_uint32), ("_pad", c_uint32)]


WAVEFRONT_MAX_BLOCKS = 64


class Wavefront(Structure):
    """userspace/gpu/nvme_ep_wavefront.h:42-47"""
    _fields_ = [("num_blocks", c_uint32), ("flags", c_uint32), ("sequence_id", c_uint64),
                ("blocks", WfBlockDesc * WAVEFRONT_MAX_BLOCKS)]


class WfCompletion(Structure):
    """userspace/gpu/nvme_ep_wavefront.h:54-60"""
    _fields_ = [("sequence_id", c_uint64), ("blocks_completed", c_uint32),
                ("blocks_failed", c_uint32), ("total_bytes", c_uint64), ("latency_ns", c_uint64)]


class Stats(Structure):
    _fields_ = [("launches", c_uint64), ("kv_bytes", c_uint64), ("errors", c_uint64),
                ("last_error", c_int), ("device", c_int), ("num_sms", c_int),
                ("last_cuda_error", c_int)]


# (name, restype, argtypes) for every symbol include/kllm_gpu.h declares.
_SIGNATURES = [
    ("kllm_gpu_create", c_void_p, []),
    ("kllm_gpu_destroy", None, [c_void_p]),
    ("kllm_gpu_get_backend", c_int, [c_void_p]),
    ("kllm_gpu_paged_attention", c_int, [c_void_p, POINTER(AttnParams)]),
    ("kllm_gpu_malloc", c_void_p, [c_void_p, c_uint64]),
    ("kllm_gpu_free", None, [c_void_p, c_void_p]),
    ("kllm_gpu_memcpy_h2d", c_int, [c_void_p, c_void_p, c_void_p, c_uint64]),
    ("kllm_gpu_get_stream", c_void_p, [c_void_p]),
    ("kllm_gpu_paged_attention_cuda", c_int,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_float,
      c_void_p]),
    ("kllm_gpu_paged_attention_v2", c_int, [c_void_p, POINTER(AttnParamsV2)]),
    ("kllm_gpu_paged_attention_v2_noalloc", c_int, [POINTER(AttnParamsV2)]),
    ("kllm_gpu_decode_workspace_size", c_uint64, [c_void_p, c_int, c_int]),
    ("kllm_gpu_kv_append_v2", c_int, [c_void_p, POINTER(KvAppendParams)]),
    ("kllm_gpu_gather_debug", c_int, [c_void_p, POINTER(GatherParams)]),
    ("kllm_gpu_prefill_v2", c_int, [c_void_p, POINTER(PrefillParams)]),
    ("kllm_gpu_table_workspace_size", c_uint64, [c_int, c_int, c_int]),
    ("kllm_gpu_build_block_tables", c_int, [c_void_p, POINTER(TableBuildParams)]),
    ("kllm_gpu_lm_head_workspace_size", c_uint64, [c_int, c_int]),
    ("kllm_gpu_lm_head_sample", c_int, [c_void_p, POINTER(LmHeadParams)]),
    ("kllm_gpu_merge_partials", c_int,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    ("kllm_gpu_memcpy_d2h", c_int, [c_void_p, c_void_p, c_void_p, c_uint64]),
    ("kllm_gpu_memcpy_h2d_async", c_int, [c_void_p, c_void_p, c_void_p, c_uint64, c_void_p]),
    ("kllm_gpu_memcpy_d2h_async", c_int, [c_void_p, c_void_p, c_void_p, c_uint64, c_void_p]),
    ("kllm_gpu_host_alloc", c_void_p, [c_void_p, c_uint64]),
    ("kllm_gpu_host_free", None, [c_void_p, c_void_p]),
    ("kllm_gpu_synchronize", c_int, [c_void_p, c_int]),
    ("kllm_gpu_get_stats", c_int, [c_void_p, POINTER(Stats)]),
    ("kllm_gpu_register_arena", c_int, [c_void_p, c_void_p, c_uint64]),
    ("kllm_gpu_clear_arenas", None, [c_void_p]),
    ("kllm_gpu_trace_enable", c_int, [c_void_p, c_int]),
    ("kllm_gpu_trace_tag", None, [c_void_p, c_uint64]),
    ("kllm_gpu_trace_read", c_int, [c_void_p, c_void_p, c_int, POINTER(c_uint64)]),
    ("kllm_gpu_comm_get_unique_id", c_int, [POINTER(c_uint8)]),
    ("kllm_gpu_comm_init", c_int, [c_void_p, c_int, c_int, POINTER(c_uint8), c_int]),
    ("kllm_gpu_comm_merge", c_int,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int]),
    ("kllm_gpu_comm_destroy", None, [c_void_p]),
    ("kllm_gpu_p2p_export", c_int, [c_void_p, c_int, c_int, POINTER(c_uint8)]),
    ("kllm_gpu_p2p_import", c_int, [c_void_p, c_int, c_int, POINTER(c_uint8)]),
    ("kllm_gpu_p2p_merge", c_int,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_int, c_void_p]),
    ("kllm_gpu_p2p_destroy", None, [c_void_p]),
]

# every symbol include/kllm_wavefront.h declares
_WF_SIGNATURES = [
    ("kllm_wavefront_create", c_void_p, [ctypes.c_char_p]),
    ("kllm_wavefront_create2", c_void_p, [ctypes.c_char_p, c_int, c_uint64, c_int]),
    ("kllm_wavefront_destroy", None, [c_void_p]),
    ("kllm_wavefront_set_index", c_int, [c_void_p, c_void_p, c_uint32, c_uint64, c_uint64]),
    ("kllm_wavefront_submit", c_int, [c_void_p, POINTER(Wavefront)]),
    ("kllm_wavefront_poll", c_int, [c_void_p, POINTER(WfCompletion), c_int]),
    ("kllm_wavefront_wait", c_int, [c_void_p, POINTER(WfCompletion), c_int, c_int]),
    ("kllm_wavefront_error", c_int, [c_void_p]),
]
WAVEFRONT_HEADER_PATH = os.path.join(os.path.dirname(HEADER_PATH), "kllm_wavefront.h")

_LIB = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Loads libkllm_gpu.so (built in-tree by ``make -C xpu-kllm_b200``)."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = path or os.environ.get("KLLM_GPU_LIB") or LIB_PATH
    if not os.path.exists(p):
        raise RuntimeError(f"libkllm_gpu.so not built: {p} (run __graft_entry__.build())")
    lib = ctypes.CDLL(p)
    for name, res, args in _SIGNATURES + _WF_SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _LIB = lib
    return lib


def symbols() -> list[str]:
    return [s[0] for s in _SIGNATURES]


def wavefront_symbols() -> list[str]:
    return [s[0] for s in _WF_SIGNATURES]


class Backend:
    """A kllm_gpu_ctx: one device, one stream, one split-KV workspace."""

    def __init__(self, lib: ctypes.CDLL | None = None):
        self.lib = lib or load()
        self.ctx = self.lib.kllm_gpu_create()
        if not self.ctx:
            raise MemoryError("kllm_gpu_create returned NULL")
        self.backend = self.lib.kllm_gpu_get_backend(self.ctx)

    def close(self):
        if self.ctx:
            self.lib.kllm_gpu_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return self.lib.kllm_gpu_get_stream(self.ctx) or 0

    def torch_stream(self):
        """The context's stream as a torch stream. Callers that mix torch ops
        with this library make it torch's current stream, so both are
        ordered on one stream (a NULL stream argument selects the context
        stream, userspace/gpu/gpu_attention.c:82, not torch's default)."""
        import torch
        return torch.cuda.ExternalStream(self.stream)

    def stats(self) -> Stats:
        s = Stats()
        self.lib.kllm_gpu_get_stats(self.ctx, ctypes.byref(s))
        return s

    def decode_v2(self, **kw) -> int:
        p = AttnParamsV2()
        p.struct_size = ctypes.sizeof(AttnParamsV2)
        for k, v in kw.items():
            setattr(p, k, v)
        return self.lib.kllm_gpu_paged_attention_v2(self.ctx, ctypes.byref(p))

    def decode_v1(self, **kw) -> int:
        p = AttnParams()
        for k, v in kw.items():
            setattr(p, k, v)
        return self.lib.kllm_gpu_paged_attention(self.ctx, ctypes.byref(p))

    def append(self, **kw) -> int:
        p = KvAppendParams()
        p.struct_size = ctypes.sizeof(KvAppendParams)
        for k, v in kw.items():
            setattr(p, k, v)
        return self.lib.kllm_gpu_kv_append_v2(self.ctx, ctypes.byref(p))

    def prefill(self, **kw) -> int:
        p = PrefillParams()
        p.struct_size = ctypes.sizeof(PrefillParams)
        for k, v in kw.items():
            setattr(p, k, v)
        return self.lib.kllm_gpu_prefill_v2(self.ctx, ctypes.byref(p))

    def gather(self, **kw) -> int:
        p = GatherParams()
        p.struct_size = ctypes.sizeof(GatherParams)
        for k, v in kw.items():
            setattr(p, k, v)
        return self.lib.kllm_gpu_gather_debug(self.ctx, ctypes.byref(p))

    def build_tables(self, **kw) -> int:
        p = TableBuildParams()
        p.struct_size = ctypes.sizeof(TableBuildParams)
        for k, v in kw.items():
            setattr(p, k, v)
        return self.lib.kllm_gpu_build_block_tables(self.ctx, ctypes.byref(p))

    def lm_head(self, **kw) -> int:
        p = LmHeadParams()
        p.struct_size = ctypes.sizeof(LmHeadParams)
        for k, v in kw.items():
            setattr(p, k, v)
        return self.lib.kllm_gpu_lm_head_sample(self.ctx, ctypes.byref(p))

    def merge(self, m, l, o, num_parts, num_rows, head_dim, out, stream=None) -> int:
        return self.lib.kllm_gpu_merge_partials(self.ctx, m, l, o, num_parts, num_rows,
                                                head_dim, out, stream)

    def synchronize(self, timeout_ms: int = 0) -> int:
        return self.lib.kllm_gpu_synchronize(self.ctx, timeout_ms)
