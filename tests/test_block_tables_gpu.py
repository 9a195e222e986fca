# SPDX-License-Identifier: Apache-2.0
"""GPU block-table build (kllm_gpu_build_block_tables) against the oracle
and the reference-made golden fixture: keys, table entries, LRU stamps,
hit/miss counts and the miss list must be bit-identical; a table built from
token ids must drive the decode kernel to the oracle's output."""
from __future__ import annotations

import os

import numpy as np
import pytest

import tablecase as tc
from tablecase import oracle

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(tc.HERE, "golden", "block_tables.npz")
BASE = 0x7f0000000000
SLOT = 1 << 20


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


def _expect(batch, entries, mb, B, total, now_ns=0, first_block=None, table=None, hashes=None):
    e = entries.copy()
    t, h, hits, misses, err = oracle.build_block_tables(
        batch.tokens, batch.starts, batch.lens, e, max_blocks=mb, block_size=B,
        arena_base=BASE, slot_bytes=SLOT, total_slots=total, k_offset=64, v_offset=4096,
        now_ns=now_ns, first_block=first_block, table=table, hashes=hashes)
    return t, h, hits, misses, err, e


def _run(be, batch, entries, mb, B, total, now_ns=0, **kw):
    d = tc.DeviceBuilder(be, batch, entries, mb, B, **kw)
    rc = d.run(arena_base=BASE, slot_bytes=SLOT, total_slots=total, k_offset=64,
               v_offset=4096, now_ns=now_ns)
    assert rc == 0, (rc, be.stats().last_cuda_error)
    return d, d.results()


def _misses(keys, entries, lens, mb, B):
    """Blocks whose key the oracle probe does not find (a hit on a slot past
    the arena is a hit with an invalid entry, not a miss)."""
    out = set()
    for s, n in enumerate(lens):
        for b in range((min(int(n), mb * B) + B - 1) // B):
            if oracle.index_probe(entries, keys[s, b].tobytes()) < 0:
                out.add((s, b))
    return out


@pytest.mark.parametrize("case", ["b16", "b16small", "b5"])
def test_golden_gpu(be, case):
    g = np.load(GOLDEN)
    B, mb, cap, total, hits, misses = (int(x) for x in g[f"{case}_meta"][:6])
    entries = g[f"{case}_entries"].reshape(-1).view(oracle.INDEX_ENTRY).copy()
    batch = tc.Batch(g[f"{case}_tokens"], g[f"{case}_starts"], g[f"{case}_lens"])
    _, r = _run(be, batch, entries, mb, B, total)
    assert r["err"] == 0
    assert (r["hashes"] == g[f"{case}_keys"]).all()
    want = tc.table_from_slots(g[f"{case}_slots"], BASE, SLOT, total, 64, 4096)
    assert (r["table"] == want).all()
    assert (r["hits"], r["misses"], r["miss_count"]) == (hits, misses, misses)
    slots = g[f"{case}_slots"]
    lens = g[f"{case}_lens"]
    want_miss = {(s, b) for s in range(len(lens)) for b in range((int(lens[s]) + B - 1) // B)
                 if slots[s, b] < 0}
    assert r["miss_list"] == want_miss
    assert (r["entries"] == entries).all()          # now_ns == 0: the index is untouched


@pytest.mark.parametrize("B", [1, 5, 16, 32, 128])
def test_random_vs_oracle(be, B):
    rng = np.random.default_rng(1000 + B)
    lens = [0, 1, 13, 14, 15, 16, 17, 29, 30, 31, 32, 33, 47, 48, 49, 700, 700, 1500, 2600]
    batch = tc.make_batch(rng, lens, shared=[(16, 15, 512), (17, 15, 333)])
    mb = 2048 // B + 1                    # the last sequence is cut: flagged
    keys = tc.all_keys(batch, B, mb)
    entries = tc.empty_index(4096)
    total = 3000
    for s, n in enumerate(lens):
        for b in range((min(n, mb * B) + B - 1) // B):
            if rng.random() < 0.55 and oracle.index_probe(entries, keys[s, b].tobytes()) < 0:
                tc.index_insert(entries, keys[s, b].tobytes(), int(rng.integers(0, total + 40)))
    for _ in range(300):                  # decoys sharing buckets
        k = bytearray(rng.integers(0, 256, 32, dtype=np.uint8).tobytes())
        k[:4] = keys[15, int(rng.integers(0, (lens[15] + B - 1) // B))].tobytes()[:4]
        tc.index_insert(entries, bytes(k), int(rng.integers(0, total)))
    t, h, hits, misses, err, e_after = _expect(batch, entries, mb, B, total, now_ns=123456789)
    _, r = _run(be, batch, entries, mb, B, total, now_ns=123456789)
    assert err == tc.ERR_SEQ_TOO_LONG and r["err"] == tc.ERR_SEQ_TOO_LONG
    assert (r["hashes"] == h).all()
    assert (r["table"] == t).all()
    assert (r["entries"] == e_after).all()         # LRU stamps on exactly the hit entries
    assert (r["hits"], r["misses"], r["miss_count"]) == (hits, misses, misses)
    assert r["miss_list"] == _misses(h, entries, lens, mb, B)


@pytest.mark.parametrize("B", [16, 5])
def test_incremental_extension(be, B):
    """Build, extend every sequence, rebuild from first_block with the same
    workspace: equal to a full build of the extended batch."""
    rng = np.random.default_rng(77 + B)
    lens1 = [0, 3, 16, 40, 257, 1000]
    grow = [5, 1, 16, 30, 300, 17]
    full = tc.make_batch(rng, [a + b for a, b in zip(lens1, grow)])
    short = tc.Batch(full.tokens, full.starts, np.array(lens1, np.int32))
    mb = (max(full.lens) + B - 1) // B + 1
    keys = tc.all_keys(full, B, mb)
    entries = tc.empty_index(2048)
    for s in range(len(lens1)):
        for b in range(0, (int(full.lens[s]) + B - 1) // B, 2):
            tc.index_insert(entries, keys[s, b].tobytes(), s * 1000 + b)
    d = tc.DeviceBuilder(be, short, entries, mb, B)
    kw = dict(arena_base=BASE, slot_bytes=SLOT, total_slots=1 << 20, k_offset=64, v_offset=4096)
    assert d.run(**kw) == 0
    r1 = d.results()
    first = [n // B for n in lens1]
    d.set_batch(full)
    assert d.run(first_block=first, **kw) == 0
    r2 = d.results()
    t_full, h_full, *_ = oracle.build_block_tables(
        full.tokens, full.starts, full.lens, entries.copy(), max_blocks=mb, block_size=B,
        total_slots=1 << 20, arena_base=BASE, slot_bytes=SLOT, k_offset=64, v_offset=4096)
    assert (r2["table"] == t_full).all()
    assert (r2["hashes"] == h_full).all()
    # only the rebuilt blocks were looked up in the second call
    nb_new = sum((int(full.lens[s]) + B - 1) // B - first[s] for s in range(len(lens1)))
    nb_old = sum((n + B - 1) // B for n in lens1)
    assert r2["hits"] + r2["misses"] == nb_old + nb_new
    assert r1["hits"] + r1["misses"] == nb_old


def test_miss_list_capacity(be):
    rng = np.random.default_rng(3)
    batch = tc.make_batch(rng, [160, 90])
    entries = tc.empty_index(16)
    _, r = _run(be, batch, entries, 10, 16, 100, miss_capacity=4)
    assert r["miss_count"] == 16 and len(r["miss_list"]) == 4
    assert r["miss_list"] <= {(s, b) for s in range(2) for b in range(10 if s == 0 else 6)}
    _, r = _run(be, batch, entries, 10, 16, 100, miss_capacity=0)
    assert r["miss_count"] == 16


def test_rejects_bad_arguments(be):
    import kllm_b200 as kb
    rng = np.random.default_rng(4)
    batch = tc.make_batch(rng, [20])
    d = tc.DeviceBuilder(be, batch, tc.empty_index(8), 4, 16)
    kw = dict(arena_base=BASE, slot_bytes=SLOT, total_slots=10, k_offset=0, v_offset=0)
    d.capacity = 6                                     # not a power of two
    assert d.run(**kw) == kb.EINVAL
    d.capacity = 8
    d.ws_bytes -= 16                                   # workspace too small
    assert d.run(**kw) == kb.ENOSPC


def test_content_addressed_decode(be):
    """C2-shaped MX-FP8 batch: index every valid page under its block key,
    build the table from token ids on the GPU, decode through it: the table
    equals the planned one and the output equals the oracle's."""
    import torch
    import kvcase
    from kllm_b200 import workloads as wl
    hc = kvcase.build_case(wl.C2, batch=16)
    c = hc.cfg
    dc = kvcase.DeviceCase(hc)
    base = dc.arena.data_ptr()
    want = wl.block_table(hc.plan, c, base, hc.valid)
    rng = np.random.default_rng(21)
    batch = tc.make_batch(rng, [int(x) for x in hc.seq_lens])
    mb = hc.plan.max_blocks
    keys = tc.all_keys(batch, c.block, mb)
    entries = tc.empty_index(1 << 14)
    for s in range(len(hc.seq_lens)):
        for b in range(mb):
            if want[s, b]["valid"]:
                tc.index_insert(entries, keys[s, b].tobytes(), int(hc.plan.slots[s, b]))
    d = tc.DeviceBuilder(be, batch, entries, mb, c.block)
    rc = d.run(arena_base=base, slot_bytes=c.slot_bytes(), total_slots=hc.plan.n_slots,
               k_offset=0, v_offset=c.page_bytes())
    assert rc == 0
    torch.cuda.synchronize()
    got = d.table.cpu().numpy().view(wl.ENTRY_DTYPE).reshape(want.shape)
    assert (got == want).all()
    out = torch.zeros((len(hc.seq_lens), c.hq, c.d), dtype=torch.int16, device="cuda")
    lens = torch.from_numpy(hc.seq_lens.astype(np.int32)).cuda()
    rc = be.decode_v2(output=out.data_ptr(), query=dc.q[0].data_ptr(),
                      block_tables=d.table.data_ptr(), seq_lens=lens.data_ptr(),
                      num_seqs=len(hc.seq_lens), num_heads=c.hq, num_kv_heads=c.hkv,
                      head_dim=c.d, max_blocks_per_seq=mb, block_size=c.block,
                      kv_dtype=c.kv_dtype, layer=0, layer_stride=c.layer_stride(),
                      scale=c.scale, split=1, stream=torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    kvcase.assert_close_bf16(out.cpu().numpy().view(np.uint16), hc.oracle_decode(),
                             what="decode through a content-addressed table")
