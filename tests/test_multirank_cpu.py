# SPDX-License-Identifier: Apache-2.0
"""The N>1 host logic on CPU ranks (gloo, world size 2): request sharding,
split-KV with an all-gather merge, and a dead rank surfacing as a bounded
error. No GPU is touched."""
from __future__ import annotations

import os
import socket
import sys
import traceback
from dataclasses import replace

import numpy as np
import pytest
import torch.multiprocessing as mp

from kllm_b200 import multigpu as mg
from kllm_b200 import workloads as wl

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    import datetime
    import torch.distributed as dist
    for p in (os.path.join(ROOT, "xpu-kllm_b200"), os.path.join(ROOT, "oracle"), HERE):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _worker(fn, rank, world, port, q):
    try:
        fn(rank, world, port, q)
    except BaseException:
        q.put((rank, "error", traceback.format_exc()))


def _run(fn, world=2, timeout=240):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(fn, r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, payload = q.get(timeout=timeout)
            results[rank] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return results


# ---- request sharding ----------------------------------------------------------

LENS6 = np.array([3000, 600, 1500, 40, 2500, 900], np.int32)


def _sharded_decode(rank, world, port, q):
    dist = _init(rank, world, port)
    import kvcase
    cfg = replace(wl.C2, batch=len(LENS6))
    mine = mg.lpt_shard(LENS6, world)[rank]
    # this rank's requests, with the data the whole batch gives them
    hc = kvcase.build_case(cfg, seq_lens=LENS6[mine], seq_ids=mine)
    out = hc.oracle_decode(q=wl.query_bf16(cfg)[mine])
    gathered = [None] * world
    dist.all_gather_object(gathered, (mine, out))
    if rank == 0:
        merged = np.zeros((len(LENS6), cfg.hq, cfg.d), np.uint16)
        for idx, o in gathered:
            merged[idx] = o
        q.put((rank, "ok", merged))
    else:
        q.put((rank, "ok", None))
    dist.destroy_process_group()


def test_request_sharding_matches_single_rank():
    import kvcase
    res = _run(_sharded_decode)
    assert all(v[0] == "ok" for v in res.values()), res
    cfg = replace(wl.C2, batch=len(LENS6))
    whole = kvcase.build_case(cfg, seq_lens=LENS6).oracle_decode()
    assert np.array_equal(res[0][1], whole)


def test_lpt_balance_on_c3():
    lens = wl.context_lengths(wl.C3)
    for n in (2, 4, 8):
        shards = mg.lpt_shard(lens, n)
        assert sorted(i for s in shards for i in s) == list(range(len(lens)))
        assert mg.imbalance(lens, shards) < 1.02, n


# ---- split-KV across ranks -------------------------------------------------------

def _split_kv(rank, world, port, q):
    import torch
    dist = _init(rank, world, port)
    import kvcase
    import oracle
    cfg = replace(wl.C4, batch=1, ctx_lo=5000, ctx_hi=5000, hq=32)
    hc = kvcase.build_case(cfg)
    c = hc.cfg
    table = hc.host_table()
    lo, hi = mg.page_ranges(hc.plan.max_blocks, world)[rank]
    t_loc, len_loc = mg.local_view(table[0], int(hc.seq_lens[0]), c.block, lo, hi)
    m, l, o = oracle.paged_decode_partials(hc.q[0], t_loc[None], np.array([len_loc], np.int32),
                                           c.hq, c.hkv, c.d, hc.plan.max_blocks, c.scale,
                                           c.block, c.kv_dtype)
    tm = [torch.zeros(c.hq) for _ in range(world)]
    tl = [torch.zeros(c.hq) for _ in range(world)]
    to = [torch.zeros(c.hq, c.d) for _ in range(world)]
    dist.all_gather(tm, torch.from_numpy(m[0]))
    dist.all_gather(tl, torch.from_numpy(l[0]))
    dist.all_gather(to, torch.from_numpy(o[0]))
    merged = mg.merge_triples(torch.stack(tm).numpy(), torch.stack(tl).numpy(),
                              torch.stack(to).numpy())
    q.put((rank, "ok", (merged, hc.oracle_decode()[0])))
    dist.destroy_process_group()


def test_split_kv_merge_matches_whole_context():
    res = _run(_split_kv)
    assert all(v[0] == "ok" for v in res.values()), res
    for rank, (_, (merged, whole)) in res.items():
        kvcase_mod = __import__("kvcase")
        kvcase_mod.assert_close_bf16(wl.f32_to_bf16(merged), whole, what=f"rank {rank}")


# ---- a rank that dies before the exchange ------------------------------------------

def _dead_peer(rank, world, port, q):
    import time
    import torch
    dist = _init(rank, world, port, timeout_s=5)
    if rank == 1:
        q.put((rank, "ok", "left"))
        q.close()
        q.join_thread()       # flush the message before leaving
        os._exit(0)           # leaves between steps, nothing in flight
    t0 = time.time()
    try:
        x = [torch.zeros(4) for _ in range(world)]
        dist.all_gather(x, torch.ones(4))
        q.put((rank, "ok", ("no error", time.time() - t0)))
    except Exception as e:   # the survivor learns of it from the group
        q.put((rank, "ok", ("error", time.time() - t0, type(e).__name__)))


def test_dead_rank_is_reported_not_hung():
    res = _run(_dead_peer, timeout=120)
    assert res[1] == ("ok", "left")
    status, payload = res[0]
    assert status == "ok" and payload[0] == "error", payload
    assert payload[1] < 60, "the survivor waited too long"


def test_merge_triples_handles_empty_parts():
    m = np.array([[0.5, -np.inf], [1.0, -np.inf]], np.float32)
    l = np.array([[2.0, 0.0], [3.0, 0.0]], np.float32)
    o = np.ones((2, 2, 4), np.float32)
    o[1] *= 3
    out = mg.merge_triples(m, l, o)
    w0, w1 = 2.0 * np.exp(0.5 - 1.0), 3.0
    assert np.allclose(out[0], (w0 * 1 + w1 * 3) / (w0 + w1))
    assert not out[1].any()
