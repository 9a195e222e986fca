# SPDX-License-Identifier: Apache-2.0
"""ctypes binding of the parity checker. TEST INFRASTRUCTURE ONLY.

Loaded only by tests/, the smoke check and bench.py's CPU-baseline leg:

* ``liboracle.so``: the C restatement (kllm_oracle.c) and the CPU harness;
* ``_ref/libkllm_ref_{avx512,scalar}.so``: the reference's own
  ``userspace/compute/ace_attention.c`` and ``mx_dequant.h`` compiled from
  its sources (oracle/Makefile), used to pin the restatement and as the
  "reference" CPU baseline;
* ``_ref/libkllm_ref_index.so``: the reference's own
  ``userspace/kvcache/cache_index.c`` with OpenSSL's ``SHA256`` block key
  (``userspace/compute/infer_gpu.c:110-118``), for the block-table build.
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
    lib.orc_sha256.restype = None
    lib.orc_sha256.argtypes = [c_void_p, ctypes.c_size_t, c_void_p]
    lib.orc_block_key.restype = None
    lib.orc_block_key.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p]
    lib.orc_index_probe.restype = ctypes.c_int64
    lib.orc_index_probe.argtypes = [c_void_p, c_uint32, c_void_p]
    lib.orc_build_block_tables.restype = c_int
    lib.orc_build_block_tables.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                           c_int, c_void_p, c_uint32, c_uint64, c_uint64,
                                           c_uint64, c_uint64, c_uint64, c_uint64, c_void_p,
                                           c_void_p, POINTER(c_uint64), POINTER(c_uint64)]
    lib.orc_lm_head_logits.restype = None
    lib.orc_lm_head_logits.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int,
                                       c_void_p]
    lib.orc_sample_greedy.restype = c_uint32
    lib.orc_sample_greedy.argtypes = [c_void_p, c_uint32]
    lib.orc_sample_temperature.restype = c_uint32
    lib.orc_sample_temperature.argtypes = [c_void_p, c_uint32, c_float, c_float]
    lib.orc_sample_top_k.restype = c_uint32
    lib.orc_sample_top_k.argtypes = [c_void_p, c_uint32, c_uint32, c_float, c_float]
    lib.orc_sample_token.restype = c_uint32
    lib.orc_sample_token.argtypes = [c_void_p, c_uint32, c_int, c_float, c_uint32, c_float]
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


_REF_INDEX = None
_REF_SAMPLING = None


def ref_sampling_lib():
    """The reference's own samplers (decode_loop.c), None when never built."""
    global _REF_SAMPLING
    if _REF_SAMPLING is None:
        p = os.path.join(REF_DIR, "libkllm_ref_sampling.so")
        if not os.path.exists(p):
            return None
        lib = ctypes.CDLL(p)
        lib.ref_sample_token.restype = c_uint32
        lib.ref_sample_token.argtypes = [c_void_p, c_uint32, c_int, c_float, c_uint32, c_float]
        lib.ref_srand.restype = None
        lib.ref_srand.argtypes = [ctypes.c_uint]
        lib.ref_rand.restype = c_int
        lib.ref_rand.argtypes = []
        _REF_SAMPLING = lib
    return _REF_SAMPLING


RAND_MAX = 2147483647


def ref_sample_with_seed(logits, method, temperature, top_k, seed):
    """The reference's sample_token with its rand() seeded; returns (token,
    r) where r is the draw the reference makes, as float32 like its
    (float)rand() / (float)RAND_MAX (decode_loop.c:95)."""
    lib = ref_sampling_lib()
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    lib.ref_srand(seed)
    x = lib.ref_rand()
    r = np.float32(np.float32(x) / np.float32(RAND_MAX))
    lib.ref_srand(seed)
    tok = lib.ref_sample_token(ptr(lg), len(lg), method, temperature, top_k, 0.0)
    return int(tok), float(r)


def ref_index_lib():
    """The reference's cache index + SHA256 block key (None when never built)."""
    global _REF_INDEX
    if _REF_INDEX is None:
        p = os.path.join(REF_DIR, "libkllm_ref_index.so")
        if not os.path.exists(p):
            return None
        lib = ctypes.CDLL(p)
        lib.ref_index_new.restype = c_void_p
        lib.ref_index_new.argtypes = [c_uint32, c_uint64]
        lib.ref_index_free.restype = None
        lib.ref_index_free.argtypes = [c_void_p]
        for name in ("ref_index_insert", "ref_index_lookup"):
            fn = getattr(lib, name)
            fn.restype = ctypes.c_int64
            fn.argtypes = [c_void_p, c_void_p]
        lib.ref_index_evict.restype = c_int
        lib.ref_index_evict.argtypes = [c_void_p, c_void_p]
        lib.ref_index_entries.restype = c_void_p
        lib.ref_index_entries.argtypes = [c_void_p]
        lib.ref_index_stats.restype = None
        lib.ref_index_stats.argtypes = [c_void_p, c_void_p]
        lib.ref_block_keys.restype = None
        lib.ref_block_keys.argtypes = [c_void_p, c_uint32, c_uint32, c_uint32, c_void_p]
        lib.ref_build_slots_mt.restype = c_int
        lib.ref_build_slots_mt.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                           c_int, c_void_p, c_void_p, c_int, POINTER(c_double)]
        lib.ref_build_slots.restype = None
        lib.ref_build_slots.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                        c_int, c_void_p]
        _REF_INDEX = lib
    return _REF_INDEX


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


# ---- content-addressed block tables -------------------------------------------

# userspace/kvcache/cache_index.h:22-27
INDEX_ENTRY = np.dtype([("hash", "u1", (32,)), ("slot_index", "<u4"), ("flags", "<u4"),
                        ("last_access_ns", "<u8")])
assert INDEX_ENTRY.itemsize == 48
INDEX_EMPTY = 0xFFFFFFFF


def sha256(msg: bytes) -> bytes:
    buf = np.frombuffer(bytes(msg), dtype=np.uint8).copy() if msg else np.zeros(1, np.uint8)
    out = np.zeros(32, dtype=np.uint8)
    orc().orc_sha256(ptr(buf), len(msg), ptr(out))
    return out.tobytes()


def block_keys(tokens: np.ndarray, seq_len: int, block_size: int, n_blocks: int,
               use_ref: bool = False) -> np.ndarray:
    """[n_blocks][32] keys of one sequence (the reference's SHA256 call when use_ref)."""
    tok = np.ascontiguousarray(tokens, dtype=np.uint32)
    if tok.size == 0:
        tok = np.zeros(1, np.uint32)
    out = np.zeros((n_blocks, 32), dtype=np.uint8)
    if use_ref:
        ref_index_lib().ref_block_keys(ptr(tok), seq_len, block_size, n_blocks, ptr(out))
    else:
        for b in range(n_blocks):
            orc().orc_block_key(ptr(tok), seq_len, block_size, b, ptr(out[b]))
    return out


def index_probe(entries: np.ndarray, key) -> int:
    e = np.ascontiguousarray(entries)
    assert e.dtype == INDEX_ENTRY
    k = np.frombuffer(bytes(key), dtype=np.uint8).copy()
    return int(orc().orc_index_probe(ptr(e), len(e), ptr(k)))


def build_block_tables(tokens, starts, seq_lens, index, *, max_blocks, block_size, arena_base,
                       slot_bytes, total_slots, k_offset, v_offset, first_block=None,
                       now_ns=0, table=None, hashes=None):
    """orc_build_block_tables; index is updated in place (LRU stamps).
    Returns (table [S][max_blocks] of 24-byte entries, hashes [S][max_blocks][32],
    hits, misses, err)."""
    tok = np.ascontiguousarray(tokens, dtype=np.uint32)
    if tok.size == 0:
        tok = np.zeros(1, np.uint32)
    st = np.ascontiguousarray(starts, dtype=np.int64)
    ln = np.ascontiguousarray(seq_lens, dtype=np.int32)
    S = len(ln)
    assert index.dtype == INDEX_ENTRY and index.flags["C_CONTIGUOUS"]
    if table is None:
        table = np.zeros(S * max_blocks * 24, dtype=np.uint8)
    if hashes is None:
        hashes = np.zeros((S, max_blocks, 32), dtype=np.uint8)
    fb = None if first_block is None else np.ascontiguousarray(first_block, dtype=np.int32)
    hits, misses = c_uint64(0), c_uint64(0)
    err = orc().orc_build_block_tables(ptr(tok), ptr(st), ptr(ln), None if fb is None else ptr(fb),
                                       S, max_blocks, block_size, ptr(index), len(index), now_ns,
                                       arena_base, slot_bytes, total_slots, k_offset, v_offset,
                                       ptr(table), ptr(hashes), ctypes.byref(hits),
                                       ctypes.byref(misses))
    return table, hashes, hits.value, misses.value, err


class RefIndex:
    """The reference's own cache index (cache_index.c) over a test arena."""

    def __init__(self, capacity: int, total_slots: int):
        self.lib = ref_index_lib()
        if self.lib is None:
            raise RuntimeError("oracle/_ref/libkllm_ref_index.so was not built")
        self.h = self.lib.ref_index_new(capacity, total_slots)
        if not self.h:
            raise ValueError("kllm_index_create rejected the capacity")
        self.capacity = capacity

    def close(self):
        if self.h:
            self.lib.ref_index_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @staticmethod
    def _key(key):
        return np.frombuffer(bytes(key), dtype=np.uint8).copy()

    def insert(self, key) -> int:
        k = self._key(key)
        return int(self.lib.ref_index_insert(self.h, ptr(k)))

    def lookup(self, key) -> int:
        k = self._key(key)
        return int(self.lib.ref_index_lookup(self.h, ptr(k)))

    def evict(self, key) -> bool:
        k = self._key(key)
        return bool(self.lib.ref_index_evict(self.h, ptr(k)))

    def entries(self) -> np.ndarray:
        """A copy of the index's entry array."""
        p = self.lib.ref_index_entries(self.h)
        raw = (ctypes.c_uint8 * (48 * self.capacity)).from_address(p)
        return np.frombuffer(bytes(raw), dtype=INDEX_ENTRY).copy()

    def stats(self) -> dict:
        out = np.zeros(6, dtype=np.uint64)
        self.lib.ref_index_stats(self.h, ptr(out))
        return dict(zip(("hits", "misses", "evictions", "insertions", "occupied", "capacity"),
                        (int(x) for x in out)))

    def build_slots(self, tokens, starts, seq_lens, max_blocks, block_size) -> np.ndarray:
        tok = np.ascontiguousarray(tokens, dtype=np.uint32)
        st = np.ascontiguousarray(starts, dtype=np.int64)
        ln = np.ascontiguousarray(seq_lens, dtype=np.int32)
        slots = np.zeros((len(ln), max_blocks), dtype=np.int64)
        self.lib.ref_build_slots(self.h, ptr(tok), ptr(st), ptr(ln), len(ln), max_blocks,
                                 block_size, ptr(slots))
        return slots

    def build_slots_mt(self, tokens, starts, seq_lens, max_blocks, block_size, nthreads):
        """(slots, keys, key_seconds, lookup_seconds) of ref_build_slots_mt."""
        tok = np.ascontiguousarray(tokens, dtype=np.uint32)
        st = np.ascontiguousarray(starts, dtype=np.int64)
        ln = np.ascontiguousarray(seq_lens, dtype=np.int32)
        slots = np.zeros((len(ln), max_blocks), dtype=np.int64)
        keys = np.zeros((len(ln), max_blocks, 32), dtype=np.uint8)
        t = (c_double * 2)()
        rc = self.lib.ref_build_slots_mt(self.h, ptr(tok), ptr(st), ptr(ln), len(ln), max_blocks,
                                         block_size, ptr(slots), ptr(keys), nthreads, t)
        assert rc == 0
        return slots, keys, t[0], t[1]


# ---- vocabulary projection and sampling ---------------------------------------

def lm_head_logits(hidden, weight, vocab_ids=None):
    """fp32 logits [rows][len(vocab_ids) or vocab] of bf16 hidden x weight^T."""
    h = np.ascontiguousarray(hidden, dtype=np.uint16)
    w = np.ascontiguousarray(weight, dtype=np.uint16)
    rows, hd = h.shape
    vocab = w.shape[0]
    ids = None if vocab_ids is None else np.ascontiguousarray(vocab_ids, dtype=np.int32)
    n = vocab if ids is None else len(ids)
    out = np.zeros((rows, n), dtype=np.float32)
    orc().orc_lm_head_logits(ptr(h), ptr(w), rows, hd, vocab, None if ids is None else ptr(ids),
                             n, ptr(out))
    return out


def sample_token(logits, method, temperature, top_k, r):
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    return int(orc().orc_sample_token(ptr(lg), len(lg), method, temperature, top_k, r))
