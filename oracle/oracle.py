# SPDX-License-Identifier: Apache-2.0
"""ctypes binding of the parity checker. TEST INFRASTRUCTURE ONLY.

Loaded only by tests/, the smoke check and bench.py's CPU-baseline leg:

* ``liboracle.so``: the C restatement (kllm_oracle.c) and the CPU harness;
* ``_ref/libkllm_ref_{avx512,scalar}.so``: the reference's own
  ``userspace/compute/ace_attention.c`` and ``mx_dequant.h`` compiled from
  its sources (oracle/Makefile), used to pin the restatement and as the
  "reference" CPU baseline.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_uint8, c_uint16, c_uint32, c_uint64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_u16p = POINTER(c_uint16)
_u8p = POINTER(c_uint8)
_f32p = POINTER(c_float)


def build(ref: str | None = None) -> None:
    """make -C oracle (the _ref libraries only where the reference exists)."""
    cmd = ["make", "-s", "-C", HERE]
    if ref:
        cmd.append(f"REF={ref}")
    subprocess.run(cmd, check=True)


def _bind(lib, prefix):
    lib.orc_bf16_to_f32.restype = c_float
    lib.orc_bf16_to_f32.argtypes = [c_uint16]
    lib.orc_f32_to_bf16.restype = c_uint16
    lib.orc_f32_to_bf16.argtypes = [c_float]
    lib.orc_e4m3_decode.restype = c_float
    lib.orc_e4m3_decode.argtypes = [c_uint8]
    lib.orc_e4m3_encode.restype = c_uint8
    lib.orc_e4m3_encode.argtypes = [c_float]
    lib.orc_mx_scale_code.restype = c_uint8
    lib.orc_mx_scale_code.argtypes = [c_float]
    lib.orc_mx_quantize_fp8.restype = None
    lib.orc_mx_quantize_fp8.argtypes = [c_void_p, c_void_p, c_void_p, c_uint32]
    lib.orc_mx_quantize_bf16_compat.restype = None
    lib.orc_mx_quantize_bf16_compat.argtypes = [c_void_p, c_void_p, c_void_p, c_uint32]
    lib.orc_attention.restype = c_int
    lib.orc_attention.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_uint32, c_uint32,
                                  c_uint32, c_uint32, c_float]
    lib.orc_gather.restype = ctypes.c_size_t
    lib.orc_gather.argtypes = [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                               c_uint64, c_void_p, c_void_p]
    lib.orc_paged_decode.restype = c_int
    lib.orc_paged_decode.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                     c_int, c_int, c_float, c_int, c_int, c_uint64, c_int]
    lib.orc_paged_decode_partials.restype = c_int
    lib.orc_paged_decode_partials.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                              c_void_p, c_int, c_int, c_int, c_int, c_int,
                                              c_float, c_int, c_int, c_uint64]
    lib.orc_merge_partials.restype = None
    lib.orc_merge_partials.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                       c_void_p]
    lib.orc_kv_append.restype = c_int
    lib.orc_kv_append.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p,
                                  c_int, c_int, c_int, c_int, c_int, c_uint64]
    lib.orc_causal_rows.restype = c_int
    lib.orc_causal_rows.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                    c_int, c_float]
    h = getattr(lib, f"{prefix}_harness_paged_decode")
    h.restype = c_int
    h.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                  c_float, c_int, c_int, c_uint64, c_int, POINTER(c_double)]
    return lib


_ORC = None
_REF = None


def orc():
    global _ORC
    if _ORC is None:
        if not os.path.exists(ORACLE_SO):
            build()
        _ORC = _bind(ctypes.CDLL(ORACLE_SO), "orc")
    return _ORC


def cpu_has_avx512_bf16() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    fl = line.split()
                    return "avx512_bf16" in fl and "avx512bw" in fl
    except OSError:
        pass
    return False


def ref_path() -> str | None:
    name = "libkllm_ref_avx512.so" if cpu_has_avx512_bf16() else "libkllm_ref_scalar.so"
    p = os.path.join(REF_DIR, name)
    return p if os.path.exists(p) else None


def ref():
    """The reference's own CPU code (None when it was never built)."""
    global _REF
    if _REF is None:
        p = ref_path()
        if p is None:
            return None
        lib = _bind(ctypes.CDLL(p), "ref")
        lib.ref_fp8_e4m3_to_f32.restype = c_float
        lib.ref_fp8_e4m3_to_f32.argtypes = [c_uint8]
        lib.ref_mx_quant_to_bf16.restype = None
        lib.ref_mx_quant_to_bf16.argtypes = [c_void_p, c_void_p, c_void_p, c_uint32]
        lib.ref_mx_dequant_bf16.restype = None
        lib.ref_mx_dequant_bf16.argtypes = [c_void_p, c_void_p, c_void_p, c_uint32]
        lib.ref_ace_probe.restype = c_int
        lib.ref_ace_probe.argtypes = []
        lib.ref_ace_attention.restype = c_int
        lib.ref_ace_attention.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_uint32,
                                          c_uint32, c_uint32, c_uint32, c_float]
        lib.ref_ace_probe()
        _REF = lib
    return _REF


def ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---- numpy-level wrappers ----------------------------------------------------

def e4m3_decode_table() -> np.ndarray:
    o = orc()
    return np.array([o.orc_e4m3_decode(c) for c in range(256)], dtype=np.float32)


def mx_quantize(x_bf16: np.ndarray):
    """[..., d] bf16 -> (payload [..., d] u8, scales [..., d/8] u8)."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    pay = np.empty(x.shape, dtype=np.uint8)
    sc = np.empty(x.shape[:-1] + (x.shape[-1] // 8,), dtype=np.uint8)
    orc().orc_mx_quantize_fp8(ptr(x), ptr(pay), ptr(sc), x.size)
    return pay, sc


def attention(q, k, v, num_heads, head_dim, seq_len, query_len, scale, use_ref=False):
    """orc_attention, or the reference's kllm_ace_attention when use_ref."""
    out = np.zeros((query_len, num_heads, head_dim), dtype=np.uint16)
    q = np.ascontiguousarray(q, dtype=np.uint16)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    fn = ref().ref_ace_attention if use_ref else orc().orc_attention
    rc = fn(ptr(q), ptr(k), ptr(v), ptr(out), num_heads, head_dim, seq_len, query_len, scale)
    if rc != 0:
        raise ValueError("attention rejected its arguments")
    return out


def paged_decode(q, table, seq_lens, hq, hkv, d, max_blocks, scale, block, kv_dtype,
                 layer_off=0, nthreads=None):
    q = np.ascontiguousarray(q, dtype=np.uint16)
    seq_lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
    out = np.zeros((len(seq_lens), hq, d), dtype=np.uint16)
    nt = nthreads or min(os.cpu_count() or 1, 32)
    rc = orc().orc_paged_decode(ptr(out), ptr(q), ptr(table), ptr(seq_lens), len(seq_lens), hq,
                                hkv, d, max_blocks, scale, block, kv_dtype, layer_off, nt)
    assert rc == 0
    return out


def paged_decode_partials(q, table, seq_lens, hq, hkv, d, max_blocks, scale, block, kv_dtype,
                          layer_off=0):
    q = np.ascontiguousarray(q, dtype=np.uint16)
    seq_lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
    S = len(seq_lens)
    m = np.zeros((S, hq), dtype=np.float32)
    l = np.zeros((S, hq), dtype=np.float32)
    o = np.zeros((S, hq, d), dtype=np.float32)
    rc = orc().orc_paged_decode_partials(ptr(m), ptr(l), ptr(o), ptr(q), ptr(table),
                                         ptr(seq_lens), S, hq, hkv, d, max_blocks, scale,
                                         block, kv_dtype, layer_off)
    assert rc == 0
    return m, l, o


def merge_partials(m, l, o):
    m = np.ascontiguousarray(m, dtype=np.float32)
    l = np.ascontiguousarray(l, dtype=np.float32)
    o = np.ascontiguousarray(o, dtype=np.float32)
    parts, rows = m.shape[0], int(np.prod(m.shape[1:]))
    d = o.shape[-1]
    out = np.zeros((rows, d), dtype=np.uint16)
    orc().orc_merge_partials(ptr(m), ptr(l), ptr(o), parts, rows, d, ptr(out))
    return out


def gather(table_row, max_blocks, seq_len, kv_head, hkv, d, block, kv_dtype, layer_off=0):
    cap = max_blocks * block
    k = np.zeros((cap + 1, d), dtype=np.uint16)
    v = np.zeros((cap + 1, d), dtype=np.uint16)
    n = orc().orc_gather(ptr(table_row), max_blocks, seq_len, kv_head, hkv, d, block, kv_dtype,
                         layer_off, ptr(k), ptr(v))
    return k[:n], v[:n]


def kv_append(k, v, tok_seq, tok_pos, table, max_blocks, hkv, d, block, kv_dtype, layer_off=0):
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    ts = np.ascontiguousarray(tok_seq, dtype=np.int32)
    tp = np.ascontiguousarray(tok_pos, dtype=np.int32)
    return orc().orc_kv_append(ptr(k), ptr(v), ptr(ts), ptr(tp), len(ts), ptr(table), max_blocks,
                               hkv, d, block, kv_dtype, layer_off)


def harness_decode(lib, prefix, q, table, seq_lens, hq, hkv, d, max_blocks, scale, block,
                   kv_dtype, layer_off=0, nthreads=1):
    """Timed multi-threaded CPU decode; returns (out, wall_s, gather_s, attn_s)."""
    q = np.ascontiguousarray(q, dtype=np.uint16)
    seq_lens = np.ascontiguousarray(seq_lens, dtype=np.int32)
    out = np.zeros((len(seq_lens), hq, d), dtype=np.uint16)
    times = (c_double * 3)()
    fn = getattr(lib, f"{prefix}_harness_paged_decode")
    rc = fn(ptr(out), ptr(q), ptr(table), ptr(seq_lens), len(seq_lens), hq, hkv, d, max_blocks,
            scale, block, kv_dtype, layer_off, nthreads, times)
    assert rc == 0
    return out, times[0], times[1], times[2]
