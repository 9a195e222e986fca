# SPDX-License-Identifier: Apache-2.0
"""Decode parity at the full shapes the throughput figures are quoted on.

C3: continuous-batching decode at Llama-3-8B attention shape, all 256
requests with log-uniform contexts in [128, 16384] (seed 0), MX-FP8 pages in
16-token blocks scattered over the arena, one layer. The cache is written on
the device by the append kernel (byte-exact to the oracle's quantizer, tested
in test_kvops_gpu.py), exactly as the benchmark writes it; the whole arena is
then copied back and the oracle decodes the same stored bytes through a host
block table.

C2: 64 requests, contexts uniform in [512, 4096], built on the host by the
seeded generator.

Tolerance (the parity contract for attention outputs): |gpu - oracle| <=
1e-3 + 2e-2 |oracle| elementwise on the bf16 outputs.
"""
from __future__ import annotations

import os
import sys
from dataclasses import replace

import numpy as np
import pytest

import kvcase
import kllm_b200 as kb
import oracle
from kllm_b200 import workloads as wl

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    b = kb.Backend()
    assert b.backend == kb.KLLM_GPU_CUDA, "libkllm_gpu found no sm_100 device"
    torch.cuda.set_stream(b.torch_stream())
    yield b
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream())
    b.close()


def test_c3_full_batch_one_layer(be):
    import torch
    import bench
    cfg = replace(wl.C3, layers=1)
    lens = wl.context_lengths(cfg, 0)
    assert len(lens) == 256 and lens.min() >= 128 and lens.max() <= 16384
    rig = bench.DecodeRig(cfg, list(range(cfg.batch)), lens, be, torch, 0, 0)
    st = torch.cuda.current_stream().cuda_stream
    rig.out.fill_(float("nan"))
    rig.launch(0, st)
    torch.cuda.synchronize()
    got = rig.out[0].view(torch.int16).cpu().numpy().view(np.uint16)

    host = rig.arena.cpu().numpy()
    table = wl.block_table(rig.plan, cfg, host.ctypes.data, slot_pitch=rig.slot_pitch)
    q = rig.q[0].view(torch.int16).cpu().numpy().view(np.uint16)
    ref = oracle.paged_decode(q, table, rig.lens, cfg.hq, cfg.hkv, cfg.d, rig.plan.max_blocks,
                              cfg.scale, cfg.block, cfg.kv_dtype, 0,
                              nthreads=os.cpu_count() or 1)
    kvcase.assert_close_bf16(got, ref, what="C3 (256 requests, layer 0)")
    # the benchmark's second layer of the step reuses the same launch path
    rig.out.fill_(float("nan"))
    rig.launch(0, st)
    torch.cuda.synchronize()
    again = rig.out[0].view(torch.int16).cpu().numpy().view(np.uint16)
    assert np.array_equal(again, got), "a repeated C3 launch differs"


def test_c2_full_batch(be):
    import torch
    hc = kvcase.build_case(wl.C2)
    assert hc.cfg.batch == 64
    dc = kvcase.DeviceCase(hc)
    dc.out.fill_(0x7FC0)
    rc = be.decode_v2(**dc.decode_kwargs(stream=torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    kvcase.assert_close_bf16(dc.out_host(), hc.oracle_decode(), what="C2 (64 requests)")
