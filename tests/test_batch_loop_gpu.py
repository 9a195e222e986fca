# SPDX-License-Identifier: Apache-2.0
"""A continuous-batching decode loop driven the way the reactor's batch step
would drive this backend (userspace/reactor/batch_scheduler.c:258-263 runs
one request per call; here one batched call per step): requests join with a
prompt, grow by one token per step and retire, their rows and arena slots
are reused. Every step: the host updates the content-addressed index (block
keys of the changed blocks, the reference's insert/evict semantics) and
mirrors it to the device, then three device calls -- incremental block-table
build, KV append (quantize-on-write) of the new tokens, batched MX-FP8 decode
-- and the output must equal the oracle's decode over a host copy of the
cache, with every block found in the index."""
from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest

import kvcase
import tablecase as tc
from tablecase import oracle

pytestmark = pytest.mark.gpu


def _evict(entries, key: bytes) -> None:
    """userspace/kvcache/cache_index.c:168-190: the entry becomes empty (no
    tombstone)."""
    pos = oracle.index_probe(entries, key)
    assert pos >= 0
    entries[pos]["slot_index"] = oracle.INDEX_EMPTY


class Loop:
    def __init__(self, be, rows=6, n_slots=160, capacity=4096, seed=0):
        import torch
        from kllm_b200 import workloads as wl
        self.torch, self.be, self.wl = torch, be, wl
        self.cfg = replace(wl.C2, batch=rows, arena_slots=None, mult_lo=None, mult_hi=None)
        c = self.cfg
        self.B = c.block
        self.rows = rows
        self.max_blocks = 40
        self.rng = np.random.default_rng(seed)
        self.host_arena = np.zeros((n_slots, c.slot_bytes()), np.uint8)
        self.dev_arena = torch.zeros(n_slots * c.slot_bytes(), dtype=torch.uint8, device="cuda")
        self.free = [int(x) for x in self.rng.permutation(n_slots)]
        self.n_slots = n_slots
        self.entries = tc.empty_index(capacity)
        self.tokens = [np.zeros(0, np.uint32) for _ in range(rows)]
        self.slots = [[] for _ in range(rows)]
        self.keys = [[] for _ in range(rows)]
        empty = tc.Batch(np.zeros(1, np.uint32), np.zeros(rows, np.int64), np.zeros(rows, np.int32))
        self.dev = tc.DeviceBuilder(be, empty, self.entries, self.max_blocks, self.B)
        self.err = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.step_no = 0

    # ---- host side (the reactor's bookkeeping) ---------------------------------
    def _key(self, r, b, n):
        return oracle.block_keys(self.tokens[r][:n], n, self.B, b + 1)[b].tobytes()

    def grow(self, r, new_tokens):
        """Appends token ids to row r; allocates pages and re-keys the blocks
        whose key changes (the old partial last block and every new one)."""
        old = len(self.tokens[r])
        self.tokens[r] = np.concatenate([self.tokens[r], new_tokens]).astype(np.uint32)
        n = len(self.tokens[r])
        first = old // self.B
        for b in range(first, (n + self.B - 1) // self.B):
            if b < len(self.keys[r]):
                _evict(self.entries, self.keys[r][b])
            else:
                self.slots[r].append(self.free.pop(0))
                self.keys[r].append(None)
            self.keys[r][b] = self._key(r, b, n)
            tc.index_insert(self.entries, self.keys[r][b], self.slots[r][b])
        return old, first

    def retire(self, r):
        for k in self.keys[r]:
            _evict(self.entries, k)
        self.free.extend(self.slots[r])
        self.tokens[r] = np.zeros(0, np.uint32)
        self.slots[r], self.keys[r] = [], []

    def host_table(self):
        c = self.cfg
        slots = np.full((self.rows, self.max_blocks), -1, np.int64)
        for r in range(self.rows):
            slots[r, :len(self.slots[r])] = self.slots[r]
        return slots, tc.table_from_slots(slots, self.host_arena.ctypes.data, c.slot_bytes(),
                                          self.n_slots, 0, c.page_bytes())

    # ---- one step: the device calls --------------------------------------------
    def step(self, growth: dict, first_block: list):
        torch, wl, c = self.torch, self.wl, self.cfg
        st = torch.cuda.current_stream().cuda_stream
        lens = np.array([len(t) for t in self.tokens], np.int32)
        packed = np.concatenate([t for t in self.tokens] + [np.zeros(1, np.uint32)])
        starts = np.concatenate([[0], np.cumsum(lens[:-1])]).astype(np.int64)
        self.dev.set_batch(tc.Batch(packed, starts, lens))
        self.dev.index.copy_(torch.from_numpy(self.entries.view(np.uint8).copy()).cuda())
        self.dev.hit_miss.zero_()
        rc = self.dev.run(arena_base=self.dev_arena.data_ptr(), slot_bytes=c.slot_bytes(),
                          total_slots=self.n_slots, k_offset=0, v_offset=c.page_bytes(),
                          first_block=first_block, hashes=False, stream=st)
        assert rc == 0, rc
        # the new tokens' K/V rows
        seq = np.concatenate([np.full(n, r, np.int32) for r, (o, n) in growth.items()])
        pos = np.concatenate([np.arange(o, o + n, dtype=np.int32)
                              for r, (o, n) in growth.items()])
        k = wl.normal_bf16(7, wl.ST_PK, self.step_no << 24, (len(seq), c.hkv, c.d))
        v = wl.normal_bf16(7, wl.ST_PV, self.step_no << 24, (len(seq), c.hkv, c.d))

        def dev(x):
            return torch.from_numpy(x.view(np.int16) if x.dtype == np.uint16 else x).cuda()
        dk, dv, dseq, dpos = dev(k), dev(v), dev(seq), dev(pos)
        rc = self.be.append(k=dk.data_ptr(), v=dv.data_ptr(), token_seq=dseq.data_ptr(),
                            token_pos=dpos.data_ptr(), num_tokens=len(seq), num_seqs=self.rows,
                            block_tables=self.dev.table.data_ptr(),
                            max_blocks_per_seq=self.max_blocks, num_kv_heads=c.hkv,
                            head_dim=c.d, block_size=self.B, kv_dtype=c.kv_dtype, layer=0,
                            layer_stride=c.layer_stride(), err_word=self.err.data_ptr(),
                            stream=st)
        assert rc == 0, rc
        q = wl.normal_bf16(7, wl.ST_Q, self.step_no << 24, (self.rows, c.hq, c.d))
        dq = dev(q)
        dlens = dev(lens)
        out = torch.zeros((self.rows, c.hq, c.d), dtype=torch.int16, device="cuda")
        rc = self.be.decode_v2(output=out.data_ptr(), query=dq.data_ptr(),
                               block_tables=self.dev.table.data_ptr(), seq_lens=dlens.data_ptr(),
                               num_seqs=self.rows, num_heads=c.hq, num_kv_heads=c.hkv,
                               head_dim=c.d, max_blocks_per_seq=self.max_blocks,
                               block_size=self.B, kv_dtype=c.kv_dtype, layer=0,
                               layer_stride=c.layer_stride(), scale=c.scale, split=1,
                               err_word=self.err.data_ptr(), stream=st)
        assert rc == 0, rc
        r = self.dev.results()
        # oracle: the same append into the host copy, then decode
        slots, htab = self.host_table()
        skipped = oracle.kv_append(k, v, seq, pos, htab, self.max_blocks, c.hkv, c.d, self.B,
                                   c.kv_dtype)
        assert skipped == 0
        want = oracle.paged_decode(q, htab, lens, c.hq, c.hkv, c.d, self.max_blocks, c.scale,
                                   self.B, c.kv_dtype)
        torch.cuda.synchronize()
        self.step_no += 1
        return r, out.cpu().numpy().view(np.uint16), want, slots, lens


def test_continuous_batching_loop(be):
    import torch
    lp = Loop(be)
    c = lp.cfg
    prompts = {0: 37, 1: 16, 2: 129, 3: 1, 4: 300}
    schedule = [("join", prompts)] + [("decode", None)] * 3 + \
        [("retire", [1, 3])] + [("decode", None)] + [("join", {1: 64, 5: 15})] + \
        [("decode", None)] * 3
    active = set()
    for kind, arg in schedule:
        growth, first = {}, [0] * lp.rows
        if kind == "retire":
            for r in arg:
                lp.retire(r)
                active.discard(r)
        for r in sorted(active):
            old, fb = lp.grow(r, lp.rng.integers(0, 128256, 1).astype(np.uint32))
            growth[r], first[r] = (old, 1), fb
        if kind == "join":
            for r, n in arg.items():
                old, fb = lp.grow(r, lp.rng.integers(0, 128256, n).astype(np.uint32))
                growth[r], first[r] = (old, n), fb
                active.add(r)
        res, got, want, slots, lens = lp.step(growth, first)
        lookups = sum((int(lens[r]) + lp.B - 1) // lp.B - first[r] for r in range(lp.rows)
                      if lens[r] > 0)
        assert res["misses"] == 0 and res["hits"] == lookups, (kind, res["hits"], lookups)
        want_tab = tc.table_from_slots(slots, lp.dev_arena.data_ptr(), c.slot_bytes(),
                                       lp.n_slots, 0, c.page_bytes())
        assert (res["table"] == want_tab).all(), f"step {lp.step_no}: table"
        assert int(lp.err.item()) == 0
        kvcase.assert_close_bf16(got, want, what=f"step {lp.step_no} ({kind})")
    # the device cache equals the oracle's, byte for byte, on every live page
    dev_arena = lp.dev_arena.cpu().numpy().reshape(lp.host_arena.shape)
    for r in sorted(active):
        for s_ in lp.slots[r]:
            assert np.array_equal(dev_arena[s_], lp.host_arena[s_]), (r, s_)
    torch.cuda.synchronize()


@pytest.fixture(scope="module")
def be():
    import torch
    import kllm_b200 as kb
    b = kb.Backend()
    assert b.backend == kb.KLLM_GPU_CUDA
    torch.cuda.set_stream(b.torch_stream())
    yield b
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream())
    b.close()
