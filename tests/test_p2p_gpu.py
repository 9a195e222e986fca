# SPDX-License-Identifier: Apache-2.0
"""Cross-GPU split-KV through the peer-memory exchange (kllm_gpu_p2p_*): two
processes, one GPU each, each decoding its half of one long context into
partial triples; the exchange-and-merge kernel must give every rank the
whole-context output of the oracle, epoch after epoch (the slot parity and
the reuse guard are exercised by several calls in a row). Skipped with
fewer than two GPUs."""
from __future__ import annotations

import os
import socket
import sys
import traceback
from dataclasses import replace

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    try:
        for p in (os.path.join(ROOT, "xpu-kllm_b200"), os.path.join(ROOT, "oracle"), HERE):
            if p not in sys.path:
                sys.path.insert(0, p)
        import ctypes
        import datetime
        import torch
        import torch.distributed as dist
        os.environ["KLLM_GPU_DEVICE"] = str(rank)
        torch.cuda.set_device(rank)
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        import kllm_b200 as kb
        import kvcase
        from kllm_b200 import multigpu as mg
        from kllm_b200 import workloads as wl

        be = kb.Backend()
        assert be.backend == kb.KLLM_GPU_CUDA
        torch.cuda.set_stream(be.torch_stream())
        cfg = replace(wl.C4, batch=1, ctx_lo=5000, ctx_hi=5000, hq=32)
        hc = kvcase.build_case(cfg)
        c = hc.cfg
        dc = kvcase.DeviceCase(hc)
        table = wl.block_table(hc.plan, c, dc.arena.data_ptr(), hc.valid)
        lo, hi = mg.page_ranges(hc.plan.max_blocks, world)[rank]
        t_loc, len_loc = mg.local_view(table[0], int(hc.seq_lens[0]), c.block, lo, hi)
        td = torch.from_numpy(t_loc[None].view(np.uint8).copy()).cuda()
        lens = torch.tensor([len_loc], dtype=torch.int32, device="cuda")
        rows = c.hq
        pm = torch.empty(rows, dtype=torch.float32, device="cuda")
        pl = torch.empty_like(pm)
        po = torch.empty((rows, c.d), dtype=torch.float32, device="cuda")
        out = torch.zeros((rows, c.d), dtype=torch.int16, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        st = torch.cuda.current_stream().cuda_stream

        h = (ctypes.c_uint8 * 64)()
        assert be.lib.kllm_gpu_p2p_export(be.ctx, rows, c.d, h) == 0
        handles = [None] * world
        dist.all_gather_object(handles, bytes(h))
        blob = b"".join(handles)
        assert be.lib.kllm_gpu_p2p_import(be.ctx, world, rank,
                                          (ctypes.c_uint8 * len(blob))(*blob)) == 0
        want = hc.oracle_decode()[0]
        for epoch in range(5):
            rc = be.decode_v2(output=None, query=dc.q[0].data_ptr(), block_tables=td.data_ptr(),
                              seq_lens=lens.data_ptr(), num_seqs=1, num_heads=c.hq,
                              num_kv_heads=c.hkv, head_dim=c.d,
                              max_blocks_per_seq=hc.plan.max_blocks, block_size=c.block,
                              kv_dtype=c.kv_dtype, layer=0, layer_stride=c.layer_stride(),
                              scale=c.scale, split=1, partial_m=pm.data_ptr(),
                              partial_l=pl.data_ptr(), partial_o=po.data_ptr(), stream=st)
            assert rc == 0, rc
            out.zero_()
            rc = be.lib.kllm_gpu_p2p_merge(be.ctx, pm.data_ptr(), pl.data_ptr(), po.data_ptr(),
                                           rows, c.d, out.data_ptr(), err.data_ptr(), 2000, st)
            assert rc == 0, rc
            torch.cuda.synchronize()
            assert int(err.item()) == 0, hex(int(err.item()))
            kvcase.assert_close_bf16(out.cpu().numpy().view(np.uint16), want,
                                     what=f"rank {rank} epoch {epoch}")
        dist.barrier()            # no rank frees its buffer while a peer may still read it
        torch.cuda.set_stream(torch.cuda.default_stream())
        be.close()
        dist.destroy_process_group()
        q.put((rank, "ok", ""))
    except BaseException:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
def test_p2p_split_kv_merge_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, status, payload = q.get(timeout=240)
            res[rank] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(v[0] == "ok" for v in res.values()), res
