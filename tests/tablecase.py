# SPDX-License-Identifier: Apache-2.0
"""Shared pieces of the block-table build tests: seeded token batches, a
cache index filled the way the reference fills it, and the device call
through the C ABI (kllm_gpu_build_block_tables)."""
from __future__ import annotations

import os
import sys
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for _p in (os.path.join(ROOT, "xpu-kllm_b200"), os.path.join(ROOT, "oracle"), HERE):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import oracle  # noqa: E402

ERR_SEQ_TOO_LONG = 0x1


def index_insert(entries: np.ndarray, key: bytes, slot: int) -> int:
    """Insertion position of userspace/kvcache/cache_index.c:141-155 (first
    empty entry probing linearly from the key's bucket), without the
    load-factor eviction; returns the position."""
    cap = len(entries)
    bucket = int.from_bytes(key[:4], "little") & (cap - 1)
    for i in range(cap):
        pos = (bucket + i) & (cap - 1)
        if entries[pos]["slot_index"] == oracle.INDEX_EMPTY:
            entries[pos]["hash"] = np.frombuffer(key, np.uint8)
            entries[pos]["slot_index"] = slot
            entries[pos]["flags"] = 0
            entries[pos]["last_access_ns"] = 1
            return pos
    raise ValueError("index full")


def empty_index(capacity: int) -> np.ndarray:
    e = np.zeros(capacity, dtype=oracle.INDEX_ENTRY)
    e["slot_index"] = oracle.INDEX_EMPTY
    return e


@dataclass
class Batch:
    tokens: np.ndarray      # uint32, packed
    starts: np.ndarray      # int64 [S]
    lens: np.ndarray        # int32 [S]

    def seq(self, s: int) -> np.ndarray:
        return self.tokens[self.starts[s]:self.starts[s] + self.lens[s]]


def make_batch(rng, lens, shared=()) -> Batch:
    """Random uint32 token ids; ``shared`` = (dst, src, n): dst's first n
    tokens equal src's."""
    seqs = [rng.integers(0, 2**32, int(n), dtype=np.uint64).astype(np.uint32) for n in lens]
    for dst, src, n in shared:
        seqs[dst][:n] = seqs[src][:n]
    toks = np.concatenate(seqs) if seqs else np.zeros(0, np.uint32)
    starts = np.cumsum([0] + [int(n) for n in lens[:-1]]).astype(np.int64)
    return Batch(toks.astype(np.uint32), starts, np.asarray(lens, np.int32))


def all_keys(batch: Batch, block_size: int, max_blocks: int) -> np.ndarray:
    """Oracle keys [S][max_blocks][32] (zero past each sequence)."""
    S = len(batch.lens)
    keys = np.zeros((S, max_blocks, 32), np.uint8)
    for s in range(S):
        n = min(int(batch.lens[s]), max_blocks * block_size)
        nb = (n + block_size - 1) // block_size
        if nb:
            keys[s, :nb] = oracle.block_keys(batch.seq(s), n, block_size, nb)
    return keys


class DeviceBuilder:
    """Device buffers for one batch shape and kllm_gpu_build_block_tables."""

    def __init__(self, be, batch: Batch, entries: np.ndarray, max_blocks: int,
                 block_size: int, miss_capacity: int | None = None):
        import torch
        self.torch = torch
        self.be = be
        S = len(batch.lens)
        self.S, self.max_blocks, self.block_size = S, max_blocks, block_size
        dev = "cuda"
        tok = batch.tokens if batch.tokens.size else np.zeros(1, np.uint32)
        self.tokens = torch.from_numpy(tok.view(np.int32).copy()).to(dev)
        self.starts = torch.from_numpy(batch.starts.copy()).to(dev)
        self.lens = torch.from_numpy(batch.lens.copy()).to(dev)
        self.index = torch.from_numpy(entries.view(np.uint8).copy()).to(dev)
        self.capacity = len(entries)
        self.table = torch.full((S * max_blocks * 24,), 0xAB, dtype=torch.uint8, device=dev)
        self.hashes = torch.full((S * max_blocks * 32,), 0xCD, dtype=torch.uint8, device=dev)
        ws = be.lib.kllm_gpu_table_workspace_size(S, max_blocks, block_size)
        self.ws_bytes = ws
        self.workspace = torch.zeros(max(ws, 16), dtype=torch.uint8, device=dev)
        self.miss_capacity = S * max_blocks if miss_capacity is None else miss_capacity
        self.miss_list = torch.full((max(self.miss_capacity, 1) * 2,), -1, dtype=torch.int32,
                                    device=dev)
        self.miss_count = torch.full((1,), -7, dtype=torch.int32, device=dev)
        self.hit_miss = torch.zeros(2, dtype=torch.int64, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        self.first = None

    def set_batch(self, batch: Batch):
        torch = self.torch
        tok = batch.tokens if batch.tokens.size else np.zeros(1, np.uint32)
        self.tokens = torch.from_numpy(tok.view(np.int32).copy()).cuda()
        self.starts = torch.from_numpy(batch.starts.copy()).cuda()
        self.lens = torch.from_numpy(batch.lens.copy()).cuda()

    def run(self, *, arena_base, slot_bytes, total_slots, k_offset, v_offset, now_ns=0,
            first_block=None, hashes=True, stream=None) -> int:
        torch = self.torch
        if first_block is not None:
            self.first = torch.from_numpy(np.asarray(first_block, np.int32).copy()).cuda()
        st = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        return self.be.build_tables(
            token_ids=self.tokens.data_ptr(), token_starts=self.starts.data_ptr(),
            seq_lens=self.lens.data_ptr(),
            first_block=self.first.data_ptr() if first_block is not None else None,
            num_seqs=self.S, max_blocks_per_seq=self.max_blocks, block_size=self.block_size,
            index=self.index.data_ptr(), index_capacity=self.capacity, now_ns=now_ns,
            arena_base=arena_base, slot_bytes=slot_bytes, total_slots=total_slots,
            k_offset=k_offset, v_offset=v_offset, block_tables=self.table.data_ptr(),
            hashes=self.hashes.data_ptr() if hashes else None,
            workspace=self.workspace.data_ptr(), workspace_bytes=self.ws_bytes,
            miss_list=self.miss_list.data_ptr() if self.miss_capacity else None,
            miss_capacity=self.miss_capacity, miss_count=self.miss_count.data_ptr(),
            hit_miss=self.hit_miss.data_ptr(), err_word=self.err.data_ptr(), stream=st)

    def results(self) -> dict:
        self.torch.cuda.synchronize()
        n = int(self.miss_count.item())
        ml = self.miss_list.cpu().numpy().reshape(-1, 2)[:min(n, self.miss_capacity)]
        return {
            "table": self.table.cpu().numpy(),
            "hashes": self.hashes.cpu().numpy().reshape(self.S, self.max_blocks, 32),
            "entries": self.index.cpu().numpy().view(oracle.INDEX_ENTRY),
            "hits": int(self.hit_miss[0].item()), "misses": int(self.hit_miss[1].item()),
            "miss_count": n, "miss_list": {(int(a), int(b)) for a, b in ml},
            "err": int(self.err.item()),
        }


def table_from_slots(slots: np.ndarray, arena_base, slot_bytes, total_slots, k_offset,
                     v_offset) -> np.ndarray:
    """24-byte entries for a slot map (-1 = miss / past the end)."""
    from kllm_b200 import workloads as wl
    t = np.zeros(slots.shape, dtype=wl.ENTRY_DTYPE)
    ok = (slots >= 0) & (slots < total_slots)
    page = np.uint64(arena_base) + slots.clip(0).astype(np.uint64) * np.uint64(slot_bytes)
    t["k"] = np.where(ok, page + np.uint64(k_offset), 0)
    t["v"] = np.where(ok, page + np.uint64(v_offset), 0)
    t["valid"] = ok.astype(np.int32)
    return t.view(np.uint8).reshape(-1)
