# SPDX-License-Identifier: Apache-2.0
"""Generates tests/golden/block_tables.npz from the REFERENCE's own code.

Run in a checkout where the reference sources exist (oracle/Makefile builds
oracle/_ref/libkllm_ref_index.so from them):

    make -C oracle && python tests/golden/make_block_table_golden.py

The index is the reference's userspace/kvcache/cache_index.c (inserts,
explicit evictions and, in the small-capacity case, its load-factor LRU
evictions), the block keys are OpenSSL's SHA256 called as
userspace/compute/infer_gpu.c:110-118 calls it, and the expected slots are
the reference's kllm_index_lookup of every block. The entry array is
snapshotted before the lookups (they only move LRU stamps). The tests run
the oracle restatement and the GPU builder on the stored inputs.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "oracle")]

import oracle  # noqa: E402

# tests/test_e2e_latency.c:141-146: the pre-warmed prompt and its key
KAT_TOKENS = [100, 200, 300, 400]


def make_case(name, block_size, capacity, total_slots, seed, with_kat):
    rng = np.random.default_rng(seed)
    lens = [0, 5, 16, 47, 300, 300, 1030]
    seqs = [rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32) for n in lens]
    seqs[5][:256] = seqs[4][:256]        # a shared 256-token prefix
    seqs[6][:160] = seqs[4][:160]        # and a shorter one
    if with_kat:
        seqs.append(np.array(KAT_TOKENS, np.uint32))
        lens.append(len(KAT_TOKENS))
    S = len(seqs)
    max_blocks = (max(lens) + block_size - 1) // block_size + 2
    tokens = np.concatenate(seqs).astype(np.uint32)
    starts = np.cumsum([0] + lens[:-1]).astype(np.int64)
    lens = np.array(lens, np.int32)

    keys = np.zeros((S, max_blocks, 32), np.uint8)
    for s in range(S):
        nb = (int(lens[s]) + block_size - 1) // block_size
        if nb:
            keys[s, :nb] = oracle.block_keys(seqs[s], int(lens[s]), block_size, nb, use_ref=True)

    idx = oracle.RefIndex(capacity, total_slots)
    distinct = {keys[s, b].tobytes() for s in range(S)
                for b in range((int(lens[s]) + block_size - 1) // block_size)}
    distinct = sorted(distinct)
    order = rng.permutation(len(distinct))
    inserted = [distinct[i] for i in order[: int(0.7 * len(distinct))]]
    decoys = [rng.integers(0, 256, 32, dtype=np.uint8).tobytes() for _ in range(40)]
    # decoys share the bucket bits of real keys, to lengthen probe chains
    for i, d in enumerate(decoys[:20]):
        decoys[i] = inserted[i % len(inserted)][:4] + d[4:]
    stream = inserted + decoys
    stream = [stream[i] for i in rng.permutation(len(stream))]
    if with_kat:
        stream.append(keys[S - 1, 0].tobytes())      # the pre-warmed prompt
    for k in stream:
        idx.insert(k)
    evicted = [inserted[i] for i in rng.choice(len(inserted), len(inserted) // 10, replace=False)]
    if with_kat:
        evicted = [k for k in evicted if k != keys[S - 1, 0].tobytes()]
    for k in evicted:
        idx.evict(k)
    entries = idx.entries()
    before = idx.stats()
    slots = idx.build_slots(tokens, starts, lens, max_blocks, block_size)
    after = idx.stats()
    idx.close()
    return {
        f"{name}_tokens": tokens, f"{name}_starts": starts, f"{name}_lens": lens,
        f"{name}_meta": np.array([block_size, max_blocks, capacity, total_slots,
                                  after["hits"] - before["hits"],
                                  after["misses"] - before["misses"],
                                  before["evictions"], before["occupied"]], np.int64),
        f"{name}_entries": entries.view(np.uint8).reshape(capacity, 48),
        f"{name}_keys": keys, f"{name}_slots": slots,
    }


def main():
    if oracle.ref_index_lib() is None:
        raise SystemExit("oracle/_ref/libkllm_ref_index.so not built: the reference sources "
                         "are needed")
    g = {}
    g.update(make_case("b16", 16, 256, 1000, 11, True))
    g.update(make_case("b16small", 16, 64, 1000, 12, False))
    g.update(make_case("b5", 5, 512, 1000, 13, False))
    np.savez_compressed(os.path.join(HERE, "block_tables.npz"), **g)
    for n in ("b16", "b16small", "b5"):
        m = g[f"{n}_meta"]
        print(n, "hits", m[4], "misses", m[5], "evictions", m[6], "occupied", m[7])


if __name__ == "__main__":
    main()
