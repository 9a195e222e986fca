# SPDX-License-Identifier: Apache-2.0
"""Seeded synthetic workloads for the paged-attention path (tests + bench).

The reference publishes no dataset for this path; every input is synthetic
and reproducible from a seed:

* values: counter-based splitmix64 -> Box-Muller in float64 -> bf16 RNE
  (the rounding of ``userspace/compute/ace_attention.c:74-80``);
* context lengths: integer-uniform or log-uniform per config;
* page placement: a random permutation of arena slots (the block table).

Page layout helpers mirror ``include/kllm_gpu.h``: a slot holds ``layers``
x (K page, V page); a page is ``num_kv_heads`` head sections of
``block_size`` token rows (plus the trailing scale bytes for MX).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

KV_BF16, KV_MX_FP8 = 0, 1

# value streams
ST_Q, ST_K, ST_V, ST_CTX, ST_PERM, ST_MULT, ST_PQ, ST_PK, ST_PV = range(1, 10)

ENTRY_DTYPE = np.dtype([("k", "<u8"), ("v", "<u8"), ("valid", "<i4"), ("pad", "<i4")])
assert ENTRY_DTYPE.itemsize == 24  # userspace/gpu/paged_attention.cu:18-22


def _mix(x: np.ndarray) -> np.ndarray:
    """splitmix64 finaliser on a uint64 array (wrapping arithmetic)."""
    with np.errstate(over="ignore"):
        z = x + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def stream_key(seed: int, stream: int) -> np.uint64:
    x = np.array([(seed * 0x100000001B3 + stream) & 0xFFFFFFFFFFFFFFFF], dtype=np.uint64)
    return _mix(x)[0]


def uniforms(key: np.uint64, idx: np.ndarray) -> np.ndarray:
    """Doubles in [0, 1), one per uint64 index."""
    return (_mix(np.uint64(key) ^ idx.astype(np.uint64)) >> np.uint64(11)).astype(
        np.float64) * (2.0 ** -53)


def normals(key: np.uint64, start: int, n: int) -> np.ndarray:
    i = np.arange(start, start + n, dtype=np.uint64)
    pair = i >> np.uint64(1)
    u1 = 1.0 - uniforms(key, pair * np.uint64(2))          # (0, 1]
    u2 = uniforms(key, pair * np.uint64(2) + np.uint64(1))
    r = np.sqrt(-2.0 * np.log(u1))
    ang = 2.0 * math.pi * u2
    return np.where((i & np.uint64(1)) == 0, r * np.cos(ang), r * np.sin(ang))


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round to nearest even (ace_attention.c:74-80 bit trick)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    with np.errstate(over="ignore"):
        b = b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))
    return (b >> np.uint32(16)).astype(np.uint16)


def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    return (np.asarray(x, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def normal_bf16(seed: int, stream: int, start: int, shape, mult=None) -> np.ndarray:
    n = int(np.prod(shape))
    z = normals(stream_key(seed, stream), start, n).reshape(shape)
    if mult is not None:
        z = z * mult
    return f32_to_bf16(z.astype(np.float32))


# ---------------------------------------------------------------------------
# configurations (shapes of the reference workload definitions)
# ---------------------------------------------------------------------------

@dataclass
class DecodeConfig:
    name: str
    batch: int
    hq: int
    hkv: int
    d: int = 128
    block: int = 16
    kv_dtype: int = KV_BF16
    ctx_kind: str = "uniform"      # uniform | loguniform | fixed
    ctx_lo: int = 64
    ctx_hi: int = 512
    layers: int = 1
    arena_slots: int | None = None  # None: 1.25 x pages needed
    mult_lo: float | None = None    # per (seq, kv head) magnitude U(lo, hi)
    mult_hi: float | None = None

    @property
    def group(self) -> int:
        return self.hq // self.hkv

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.d)

    def section_bytes(self) -> int:
        if self.kv_dtype == KV_MX_FP8:
            return self.block * self.d + self.block * (self.d // 8)
        return self.block * self.d * 2

    def page_bytes(self) -> int:        # one of K / V, one layer
        return self.hkv * self.section_bytes()

    def layer_stride(self) -> int:      # K and V of one layer
        return 2 * self.page_bytes()

    def slot_bytes(self) -> int:
        return self.layers * self.layer_stride()

    def kv_bytes_per_token(self) -> int:  # per layer, K + V, algorithmic
        el = 1 if self.kv_dtype == KV_MX_FP8 else 2
        sc = self.d // 8 if self.kv_dtype == KV_MX_FP8 else 0
        return self.hkv * 2 * (self.d * el + sc)


C1 = DecodeConfig("c1_bf16_b8_ctx64-512", batch=8, hq=32, hkv=8, kv_dtype=KV_BF16,
                  ctx_kind="uniform", ctx_lo=64, ctx_hi=512, arena_slots=512)
C2 = DecodeConfig("c2_mxfp8_b64_ctx512-4096", batch=64, hq=32, hkv=8, kv_dtype=KV_MX_FP8,
                  ctx_kind="uniform", ctx_lo=512, ctx_hi=4096, mult_lo=0.5, mult_hi=4.0)
C3 = DecodeConfig("c3_mxfp8_llama3-8b_b256_l32_ctx128-16384", batch=256, hq=32, hkv=8,
                  kv_dtype=KV_MX_FP8, ctx_kind="loguniform", ctx_lo=128, ctx_hi=16384,
                  layers=32, mult_lo=0.5, mult_hi=4.0)
C4 = DecodeConfig("c4_mxfp8_b1_ctx131072_64q8kv", batch=1, hq=64, hkv=8, kv_dtype=KV_MX_FP8,
                  ctx_kind="fixed", ctx_lo=131072, ctx_hi=131072, mult_lo=0.5, mult_hi=4.0)
CONFIGS = {c.name: c for c in (C1, C2, C3, C4)}

# Chunked prefill + KV append: 16 prompts of 2048 tokens, BF16 Q/K/V ~ N(0,1),
# written into an MX-FP8 cache; the first quarter of the prompts share a
# 1024-token prefix chain already in the cache (content-addressed hits), so
# they prefill only their last 1024 tokens over those shared pages.
C5 = DecodeConfig("c5_prefill_b16_2048_mxfp8_prefix1024", batch=16, hq=32, hkv=8,
                  kv_dtype=KV_MX_FP8, ctx_kind="fixed", ctx_lo=2048, ctx_hi=2048)
C5_SHARED_PREFIX = 1024
PREFILL_CONFIGS = {C5.name: C5}


# Content-addressed block-table builds (token ids -> block keys -> index
# probe -> table). "warm": every block of every request is in the index (a
# decode batch whose pages are all resident); "prefix": only the shared
# prefix chain is (prompt admission with prefix reuse, the rest misses).
VOCAB = 128256                     # Llama-3 token id range


@dataclass(frozen=True)
class TableConfig:
    name: str
    lengths: DecodeConfig          # requests and context lengths
    warm: str                      # "all" | "prefix"
    index_capacity: int            # power of two


T3 = TableConfig("t3_tables_b256_ctx128-16384_warm", C3, "all", 1 << 17)
T5 = TableConfig("t5_tables_b16_2048_prefix1024", C5, "prefix", 1 << 12)
TABLE_CONFIGS = {t.name: t for t in (T3, T5)}


# KV block arrival into VRAM (the wavefront path): `blocks` records of
# `record_bytes` (one 16-token MX-FP8 K+V page pair of one layer: 2 x 8 kv
# heads x (16 x 128 + 16 x 16) bytes) fetched by key from a store file, in
# wavefronts of 64 blocks.
@dataclass(frozen=True)
class ArrivalConfig:
    name: str
    blocks: int
    record_bytes: int
    staging: int                   # page-locked staging buffers


# Vocabulary projection + sampling (the step after attention): Llama-3-8B
# shapes, bf16 weights ~ N(0, 1/hidden) x 1.5, hidden ~ N(0, 1).
@dataclass(frozen=True)
class LmHeadConfig:
    name: str
    rows: int
    hidden: int
    vocab: int
    sampling: str                  # "greedy" | "mixed" (temperature / top-k / top-p rows)


L3 = LmHeadConfig("l3_lm_head_llama3-8b_b256_greedy", 256, 4096, 128256, "greedy")
L3S = LmHeadConfig("l3_lm_head_llama3-8b_b256_sampled", 256, 4096, 128256, "mixed")
LM_HEAD_CONFIGS = {c.name: c for c in (L3, L3S)}


W3 = ArrivalConfig("w3_kv_arrival_4096x36k", 4096, 36864, 8)
ARRIVAL_CONFIGS = {W3.name: W3}


def table_tokens(tc: TableConfig, seed: int = 0):
    """(tokens uint32 packed, starts int64, lens int32): seeded token ids in
    [0, VOCAB); for the prefix workload the prompts with a cached context
    share its tokens (so their first blocks have the same keys)."""
    cfg = tc.lengths
    rng = np.random.default_rng([seed, 0x7AB1E])
    if tc.warm == "prefix":
        ctx, chunk = prefill_split(cfg)
        lens = (ctx + chunk).astype(np.int32)
        seqs = [rng.integers(0, VOCAB, int(n)).astype(np.uint32) for n in lens]
        shared = rng.integers(0, VOCAB, int(ctx.max())).astype(np.uint32)
        for s in range(len(lens)):
            if ctx[s]:
                seqs[s][:ctx[s]] = shared[:ctx[s]]
    else:
        lens = context_lengths(cfg, seed).astype(np.int32)
        seqs = [rng.integers(0, VOCAB, int(n)).astype(np.uint32) for n in lens]
    tokens = np.concatenate(seqs).astype(np.uint32)
    starts = np.concatenate([[0], np.cumsum(lens[:-1], dtype=np.int64)]).astype(np.int64)
    return tokens, starts, lens


def prefill_split(cfg: DecodeConfig, shared_prefix: int = C5_SHARED_PREFIX):
    """(cached context, chunk length) per prompt: the first batch/4 prompts
    hit the shared prefix chain."""
    n_hit = cfg.batch // 4
    ctx = np.zeros(cfg.batch, np.int32)
    ctx[:n_hit] = shared_prefix
    chunk = np.full(cfg.batch, cfg.ctx_lo, np.int32) - ctx
    return ctx, chunk


def prefill_flops(ctx: np.ndarray, chunk: np.ndarray, hq: int, d: int) -> int:
    """Causal attention FLOPs (QK^T and PV, 2 each per multiply-add): chunk
    row j of a prompt attends to ctx + j + 1 keys."""
    keys = 0
    for c0, n in zip(ctx.tolist(), chunk.tolist()):
        keys += n * c0 + n * (n + 1) // 2
    return 4 * d * hq * keys


def plan_prefill_pages(cfg: DecodeConfig, ctx: np.ndarray, chunk: np.ndarray, seed: int = 0,
                       n_slots: int | None = None) -> PagePlan:
    """Pages of every prompt; prompts with a cached context share one chain
    of pages for it (the first prompt's), as content-addressed hits do."""
    total = ctx + chunk
    plan = plan_pages(cfg, total, seed, n_slots=n_slots)
    hits = [s for s in range(len(ctx)) if ctx[s] > 0]
    if hits:
        npg = int(ctx[hits[0]]) // cfg.block
        for s in hits[1:]:
            assert int(ctx[s]) == int(ctx[hits[0]])
            plan.slots[s, :npg] = plan.slots[hits[0], :npg]
    return plan


def context_lengths(cfg: DecodeConfig, seed: int = 0) -> np.ndarray:
    u = uniforms(stream_key(seed, ST_CTX), np.arange(cfg.batch, dtype=np.uint64))
    if cfg.ctx_kind == "fixed":
        return np.full(cfg.batch, cfg.ctx_lo, dtype=np.int32)
    if cfg.ctx_kind == "uniform":
        n = cfg.ctx_hi - cfg.ctx_lo + 1
        return (cfg.ctx_lo + np.floor(u * n)).astype(np.int32)
    lo, hi = math.log(cfg.ctx_lo), math.log(cfg.ctx_hi)
    return np.clip(np.rint(np.exp(lo + u * (hi - lo))), cfg.ctx_lo, cfg.ctx_hi).astype(np.int32)


def magnitudes(cfg: DecodeConfig, seed: int = 0) -> np.ndarray | None:
    """Per (seq, kv head) multiplier, U(mult_lo, mult_hi)."""
    if cfg.mult_lo is None:
        return None
    u = uniforms(stream_key(seed, ST_MULT), np.arange(cfg.batch * cfg.hkv, dtype=np.uint64))
    return (cfg.mult_lo + u * (cfg.mult_hi - cfg.mult_lo)).reshape(cfg.batch, cfg.hkv)


def permutation(n: int, seed: int, salt: int = 0) -> np.ndarray:
    keys = _mix(np.uint64(stream_key(seed, ST_PERM) ^ np.uint64(salt)) ^
                np.arange(n, dtype=np.uint64))
    return np.argsort(keys, kind="stable").astype(np.int64)


@dataclass
class PagePlan:
    """Which arena slot holds page b of sequence s (-1: no page)."""
    seq_lens: np.ndarray
    slots: np.ndarray          # int64 [batch, max_blocks]
    n_slots: int
    max_blocks: int
    pages_used: int = field(default=0)


def plan_pages(cfg: DecodeConfig, seq_lens: np.ndarray, seed: int = 0,
               max_blocks: int | None = None, n_slots: int | None = None) -> PagePlan:
    pages = (seq_lens.astype(np.int64) + cfg.block - 1) // cfg.block
    need = int(pages.sum())
    mb = max_blocks or max(1, int(pages.max()) if len(pages) else 1)
    total = n_slots or cfg.arena_slots or max(need, int(math.ceil(need * 1.25)))
    if total < need:
        raise ValueError(f"arena of {total} slots < {need} pages needed")
    perm = permutation(total, seed)
    slots = np.full((len(seq_lens), mb), -1, dtype=np.int64)
    nxt = 0
    for s, p in enumerate(pages):
        slots[s, :p] = perm[nxt:nxt + p]
        nxt += p
    return PagePlan(seq_lens=seq_lens.astype(np.int32), slots=slots, n_slots=total,
                    max_blocks=mb, pages_used=need)


def block_table(plan: PagePlan, cfg: DecodeConfig, base: int, valid=None,
                slot_pitch: int | None = None) -> np.ndarray:
    """Entries {k_ptr, v_ptr, valid} for an arena at address ``base``.
    ``slot_pitch``: bytes between consecutive slots (default: a slot holds
    every layer, ``cfg.slot_bytes()``; a layer-major arena passes
    ``cfg.layer_stride()`` and a layer stride of n_slots x that)."""
    t = np.zeros(plan.slots.shape, dtype=ENTRY_DTYPE)
    used = plan.slots >= 0
    pitch = cfg.slot_bytes() if slot_pitch is None else slot_pitch
    addr = np.uint64(base) + plan.slots.clip(0).astype(np.uint64) * np.uint64(pitch)
    t["k"] = np.where(used, addr, 0)
    t["v"] = np.where(used, addr + np.uint64(cfg.page_bytes()), 0)
    t["valid"] = used.astype(np.int32) if valid is None else (used & valid).astype(np.int32)
    return t


def kv_elem_index(s: int, t0: int, hkv: int, d: int) -> int:
    """First stream index of token t0 of sequence s ([s][t][h][d] order)."""
    return ((s << 24) + t0) * hkv * d


def seq_kv_bf16(cfg: DecodeConfig, s: int, ntok: int, seed: int = 0, layer: int = 0,
                mult: np.ndarray | None = None):
    """K, V of sequence s as bf16 [ntok, hkv, d] (token-major, the reference's
    [token][kv_head][dim] order, userspace/kvcache/block_format.h:101-120)."""
    m = None if mult is None else mult[s][None, :, None]
    start = kv_elem_index(s, 0, cfg.hkv, cfg.d) + (layer << 50)
    k = normal_bf16(seed, ST_K, start, (ntok, cfg.hkv, cfg.d), m)
    v = normal_bf16(seed, ST_V, start, (ntok, cfg.hkv, cfg.d), m)
    return k, v


def query_bf16(cfg: DecodeConfig, seed: int = 0, layer: int = 0) -> np.ndarray:
    return normal_bf16(seed, ST_Q, layer << 50, (cfg.batch, cfg.hq, cfg.d))


def algorithmic_bytes(cfg: DecodeConfig, seq_lens: np.ndarray, layers: int | None = None) -> int:
    """KV bytes (each counted once) + Q/O + block table + seq_lens of one step."""
    nl = cfg.layers if layers is None else layers
    tokens = int(np.maximum(seq_lens, 0).sum())
    blocks = int(((np.maximum(seq_lens, 0) + cfg.block - 1) // cfg.block).sum())
    kv = tokens * cfg.kv_bytes_per_token() * nl
    qo = len(seq_lens) * cfg.hq * cfg.d * 2 * 2 * nl
    return kv + qo + (blocks * 24 + len(seq_lens) * 4) * nl
