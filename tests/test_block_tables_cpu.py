# SPDX-License-Identifier: Apache-2.0
"""Content-addressed block tables on the CPU: the oracle's SHA-256, block
keys, index probe and table build, pinned against Python's hashlib, the
reference's own OpenSSL SHA256 call (userspace/compute/infer_gpu.c:110-118),
the reference's own cache index (userspace/kvcache/cache_index.c, compiled
into oracle/_ref) and the golden fixture that build produced."""
from __future__ import annotations

import hashlib
import os
import re
import struct

import numpy as np
import pytest

import tablecase as tc
from tablecase import oracle

GOLDEN = os.path.join(tc.HERE, "golden", "block_tables.npz")
needs_ref = pytest.mark.skipif(oracle.ref_index_lib() is None,
                               reason="reference index library not built")


def _primes(n):
    ps, x = [], 2
    while len(ps) < n:
        if all(x % p for p in ps):
            ps.append(x)
        x += 1
    return ps


def _iroot(v, k):
    lo, hi = 0, 1
    while hi ** k <= v:
        hi *= 2
    while hi - lo > 1:
        m = (lo + hi) // 2
        lo, hi = (m, hi) if m ** k <= v else (lo, m)
    return lo


def test_sha256_round_constants_in_sources():
    """FIPS 180-4 4.2.2: K_t = first 32 fractional bits of cbrt(prime_t),
    recomputed exactly and compared with both source files' tables."""
    want = [_iroot(p << 96, 3) & 0xFFFFFFFF for p in _primes(64)]
    iv = [_iroot(p << 64, 2) & 0xFFFFFFFF for p in _primes(8)]
    for rel in ("xpu-kllm_b200/csrc/block_tables.cu", "oracle/content_index.c"):
        src = open(os.path.join(tc.ROOT, rel)).read()
        k_block = re.search(r"(?:kShaK|sha_k)\[64\]\s*=\s*\{([^}]*)\}", src).group(1)
        got = [int(x, 16) for x in re.findall(r"0x([0-9a-f]{8})u", k_block)]
        assert got == want, rel
        got_iv = [int(x, 16) for x in re.findall(r"0x([0-9a-f]{8})u", src)
                  if int(x, 16) in iv]
        assert set(got_iv) == set(iv), rel


def test_sha256_vs_hashlib():
    rng = np.random.default_rng(0)
    assert oracle.sha256(b"abc").hex() == hashlib.sha256(b"abc").hexdigest()
    assert oracle.sha256(b"") == hashlib.sha256(b"").digest()
    for n in list(range(0, 200)) + [447, 448, 511, 512, 4093, 65536]:
        m = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert oracle.sha256(m) == hashlib.sha256(m).digest(), n


@pytest.mark.parametrize("block_size", [1, 5, 16, 128])
def test_block_keys_vs_hashlib(block_size):
    rng = np.random.default_rng(block_size)
    tok = rng.integers(0, 2**32, 333, dtype=np.uint64).astype(np.uint32)
    nb = (333 + block_size - 1) // block_size
    keys = oracle.block_keys(tok, 333, block_size, nb)
    for b in range(nb):
        n = min((b + 1) * block_size, 333)
        assert keys[b].tobytes() == hashlib.sha256(tok[:n].astype("<u4").tobytes()).digest()


@needs_ref
@pytest.mark.parametrize("block_size", [1, 5, 16, 128])
def test_block_keys_vs_reference_call(block_size):
    rng = np.random.default_rng(100 + block_size)
    for n in (0, 1, 15, 16, 17, 400):
        tok = rng.integers(0, 2**32, max(n, 1), dtype=np.uint64).astype(np.uint32)[:n]
        nb = (n + block_size - 1) // block_size
        a = oracle.block_keys(tok, n, block_size, nb)
        b = oracle.block_keys(tok, n, block_size, nb, use_ref=True)
        assert (a == b).all(), (n, block_size)


def test_kat_prewarmed_prompt_key():
    """tests/test_e2e_latency.c:141-146: the pre-warmed prompt {100, 200, 300,
    400} is keyed by SHA-256 of its 16 little-endian bytes."""
    toks = np.array([100, 200, 300, 400], np.uint32)
    want = hashlib.sha256(struct.pack("<4I", 100, 200, 300, 400)).digest()
    assert oracle.block_keys(toks, 4, 16, 1)[0].tobytes() == want
    g = np.load(GOLDEN)
    S = len(g["b16_lens"])
    assert g["b16_keys"][S - 1, 0].tobytes() == want
    assert g["b16_slots"][S - 1, 0] >= 0        # inserted, then found by the reference


@needs_ref
@pytest.mark.parametrize("capacity", [1, 2, 8, 64, 256])
def test_probe_vs_reference_index(capacity):
    """Random inserts (with the reference's load-factor LRU eviction) and
    explicit evictions on the reference's index; the oracle probe over its
    entry array must find exactly what kllm_index_lookup finds, including
    the entries an eviction cut off from their bucket."""
    rng = np.random.default_rng(capacity)
    idx = oracle.RefIndex(capacity, 4 * capacity + 10)
    keys = [rng.integers(0, 256, 32, dtype=np.uint8).tobytes() for _ in range(3 * capacity + 5)]
    for k in keys[: 2 * capacity]:
        idx.insert(k)
    for i in rng.choice(2 * capacity, capacity // 2, replace=False):
        idx.evict(keys[i])
    for k in keys[2 * capacity: 2 * capacity + capacity // 4]:
        idx.insert(k)
    e = idx.entries()
    for k in keys:
        pos = oracle.index_probe(e, k)
        want = idx.lookup(k)
        assert want == (-1 if pos < 0 else int(e[pos]["slot_index"]))


@pytest.mark.parametrize("case", ["b16", "b16small", "b5"])
def test_golden_oracle(case):
    """The oracle build on the fixture's inputs reproduces the reference's
    keys, lookups and hit/miss counts."""
    g = np.load(GOLDEN)
    B, mb, cap, total, hits, misses = (int(x) for x in g[f"{case}_meta"][:6])
    entries = g[f"{case}_entries"].reshape(-1).view(oracle.INDEX_ENTRY).copy()
    base, sb = 0x7f0000000000, 1 << 20
    table, hashes, h, m, err = oracle.build_block_tables(
        g[f"{case}_tokens"], g[f"{case}_starts"], g[f"{case}_lens"], entries,
        max_blocks=mb, block_size=B, arena_base=base, slot_bytes=sb, total_slots=total,
        k_offset=64, v_offset=4096)
    assert err == 0
    assert (hashes == g[f"{case}_keys"]).all()
    assert (table == tc.table_from_slots(g[f"{case}_slots"], base, sb, total, 64, 4096)).all()
    assert (h, m) == (hits, misses)


@needs_ref
def test_oracle_build_vs_reference_path():
    """Random batch with shared prefixes: the oracle build's slots equal the
    reference's per-block SHA256 + kllm_index_lookup path."""
    rng = np.random.default_rng(5)
    lens = [0, 1, 13, 14, 15, 16, 17, 31, 32, 33, 500, 500, 900]
    batch = tc.make_batch(rng, lens, shared=[(11, 10, 400), (12, 10, 96)])
    B, mb = 16, 60
    keys = tc.all_keys(batch, B, mb)
    idx = oracle.RefIndex(1024, 5000)
    for s in range(len(lens)):
        for b in range((lens[s] + B - 1) // B):
            if rng.random() < 0.6:
                idx.insert(keys[s, b].tobytes())
    entries = idx.entries()
    want = idx.build_slots(batch.tokens, batch.starts, batch.lens, mb, B)
    table, hashes, h, m, err = oracle.build_block_tables(
        batch.tokens, batch.starts, batch.lens, entries.copy(), max_blocks=mb, block_size=B,
        arena_base=1 << 40, slot_bytes=4096, total_slots=5000, k_offset=0, v_offset=2048)
    assert (table == tc.table_from_slots(want, 1 << 40, 4096, 5000, 0, 2048)).all()
    assert (hashes == keys).all()


def test_oracle_flags_and_stamps():
    """Past-the-end entries are zero, a too-long sequence is cut and
    flagged, hits stamp last_access_ns, slots past the arena give invalid
    entries."""
    rng = np.random.default_rng(9)
    batch = tc.make_batch(rng, [40, 100])
    B, mb = 16, 4                      # sequence 1 (100 tokens) exceeds 4 x 16
    keys = tc.all_keys(batch, B, mb)
    e = tc.empty_index(64)
    tc.index_insert(e, keys[0, 0].tobytes(), 3)
    tc.index_insert(e, keys[0, 2].tobytes(), 99)     # beyond total_slots
    tc.index_insert(e, keys[1, 3].tobytes(), 7)      # key of the cut prefix (64 tokens)
    table, hashes, h, m, err = oracle.build_block_tables(
        batch.tokens, batch.starts, batch.lens, e, max_blocks=mb, block_size=B,
        arena_base=1 << 32, slot_bytes=256, total_slots=50, k_offset=0, v_offset=128,
        now_ns=777)
    assert err == 1
    slots = np.full((2, mb), -1)
    slots[0, 0], slots[1, 3] = 3, 7
    assert (table == tc.table_from_slots(slots, 1 << 32, 256, 50, 0, 128)).all()
    assert (h, m) == (3, 4)                          # 3 blocks of seq 0 + 4 of seq 1
    assert sorted(e["last_access_ns"][e["slot_index"] != oracle.INDEX_EMPTY]) == [777] * 3
    assert (hashes[0, 3] == 0).all()                 # past the end of sequence 0
