# SPDX-License-Identifier: Apache-2.0
"""kllm_gpu_paged_attention_v2_noalloc: the decode entry point for callers
that may not allocate device memory (for instance a polling reactor thread
under a zero-allocation rule, where cudaMalloc can stall or fail once the KV
arena owns the GPU). It keeps its split-KV scratch in a fixed array inside
the library instead of a context workspace.

Checked through the C ABI against kllm_gpu_paged_attention_v2 on two calls in
a row (the second call runs on scratch the first one left behind), with the
same tolerance as the other parity tests; also the partial-triple outputs,
more sequences than one launch takes (the chunk loop), a context long enough
to queue its segments for the wide merge, split < 0, and the documented
start-up order (a zero-work call per device, then the arena fills the GPU).
This file is collected last so that a run stopping at its first failure has
run every other test first.
"""
from __future__ import annotations

import ctypes
from dataclasses import replace

import numpy as np
import pytest

import kvcase
import kllm_b200 as kb
from kllm_b200 import workloads as wl

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    import torch
    assert torch.cuda.is_available()
    b = kb.Backend(kb.load())
    assert b.backend == kb.KLLM_GPU_CUDA
    torch.cuda.set_stream(b.torch_stream())
    yield b
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream())
    b.close()


def _params(dc, be, **over) -> kb.AttnParamsV2:
    p = kb.AttnParamsV2()
    p.struct_size = ctypes.sizeof(p)
    for k, v in dc.decode_kwargs(stream=be.stream, **over).items():
        setattr(p, k, v)
    return p


def _noalloc(be, p) -> int:
    return be.lib.kllm_gpu_paged_attention_v2_noalloc(ctypes.byref(p))


def _context_entry(be, dc, **over):
    assert be.decode_v2(**dc.decode_kwargs(stream=be.stream, **over)) == 0
    return dc.out_host().copy()


def test_zero_work_setup_then_call_with_device_memory_nearly_full(be):
    """The start-up order the header documents: one call with num_seqs == 0
    per device (it loads the scratch and the decode code), then the KV arena
    takes nearly all device memory, then the decode calls allocate nothing."""
    import torch
    cfg = replace(wl.C2, mult_lo=0.5, mult_hi=4.0)
    hc = kvcase.build_case(cfg, batch=8)
    dc = kvcase.DeviceCase(hc)
    ref = _context_entry(be, dc)
    dc.out.fill_(0x7FC0)
    assert _noalloc(be, _params(dc, be, num_seqs=0)) == 0
    free, _ = torch.cuda.mem_get_info()
    filler = torch.empty(max(0, free - (1 << 30)), dtype=torch.uint8, device="cuda")
    try:
        for _ in range(2):
            assert _noalloc(be, _params(dc, be)) == 0
        torch.cuda.synchronize()
    finally:
        del filler
        torch.cuda.empty_cache()
    kvcase.assert_close_bf16(dc.out_host(), ref, what="no-alloc with memory nearly full")


@pytest.mark.parametrize("kv", [wl.KV_MX_FP8, wl.KV_BF16])
def test_noalloc_matches_context_entry_point_twice(be, kv):
    cfg = replace(wl.C2, kv_dtype=kv, mult_lo=0.5, mult_hi=4.0)
    hc = kvcase.build_case(cfg, batch=8)
    dc = kvcase.DeviceCase(hc)
    ref = _context_entry(be, dc)
    kvcase.assert_close_bf16(ref, hc.oracle_decode(), what="context entry point")

    outs = []
    for _ in range(2):
        dc.out.fill_(0x7FC0)   # NaN: every element must be written
        assert _noalloc(be, _params(dc, be)) == 0
        outs.append(dc.out_host().copy())
    for i, got in enumerate(outs):
        kvcase.assert_close_bf16(got, ref, what=f"no-alloc call {i + 1}")
    assert np.array_equal(outs[0], outs[1]), "second call differs from the first"

    # sizes beyond the scratch's counter capacity are refused up front
    p = _params(dc, be)
    p.num_seqs = 65536 // cfg.hkv + 1
    assert _noalloc(be, p) == kb.ENOSPC
    # a table longer than 2^30 tokens per sequence is refused, as v2 does
    p = _params(dc, be)
    p.max_blocks_per_seq = (1 << 30) // cfg.block + 1
    assert _noalloc(be, p) == kb.EINVAL


def test_noalloc_partial_triples_match_context_entry_point(be):
    import torch
    cfg = replace(wl.C2, mult_lo=0.5, mult_hi=4.0)
    hc = kvcase.build_case(cfg, seq_lens=[3000, 17, 0, 1, 900, 4096])
    dc = kvcase.DeviceCase(hc)
    rows = hc.cfg.batch * cfg.hq

    def triples():
        return (torch.full((rows,), float("nan"), device="cuda"),
                torch.full((rows,), float("nan"), device="cuda"),
                torch.full((rows, cfg.d), float("nan"), device="cuda"))

    def ptrs(t):
        return dict(output=None, partial_m=t[0].data_ptr(), partial_l=t[1].data_ptr(),
                    partial_o=t[2].data_ptr())
    ref = triples()
    assert be.decode_v2(**dc.decode_kwargs(stream=be.stream, **ptrs(ref))) == 0
    for call in range(2):
        got = triples()
        assert _noalloc(be, _params(dc, be, **ptrs(got))) == 0
        torch.cuda.synchronize()
        for name, g, r in zip("mlo", got, ref):
            kvcase.assert_close_f32(g.cpu().numpy(), r.cpu().numpy(),
                                    what=f"partial {name}, call {call + 1}")


def test_noalloc_more_sequences_than_one_launch(be):
    """4,500 short sequences: the entry point cuts them into launches of
    4,096, each with its own counters in the shared scratch."""
    cfg = replace(wl.C2, hq=8, hkv=2, mult_lo=0.5, mult_hi=4.0, arena_slots=None)
    lens = (np.arange(4500) * 7 % 37).astype(np.int32)       # 0 .. 36 tokens
    hc = kvcase.build_case(cfg, seq_lens=lens, max_blocks=3)
    dc = kvcase.DeviceCase(hc)
    ref = _context_entry(be, dc)
    kvcase.assert_close_bf16(ref, hc.oracle_decode(), what="context entry point")
    for call in range(2):
        dc.out.fill_(0x7FC0)
        assert _noalloc(be, _params(dc, be)) == 0
        kvcase.assert_close_bf16(dc.out_host(), ref, what=f"4,500 sequences, call {call + 1}")


def test_noalloc_long_context_wide_merge(be):
    """One 48,000-token context: each segment spans hundreds of warps, so it
    is queued for the wide-merge kernel, whose queue header lives in the
    shared scratch."""
    cfg = replace(wl.C2, hq=8, hkv=2, mult_lo=0.5, mult_hi=4.0, arena_slots=None)
    hc = kvcase.build_case(cfg, seq_lens=[48000])
    dc = kvcase.DeviceCase(hc)
    ref = _context_entry(be, dc)
    kvcase.assert_close_bf16(ref, hc.oracle_decode(), what="context entry point")
    for call in range(2):
        dc.out.fill_(0x7FC0)
        assert _noalloc(be, _params(dc, be)) == 0
        kvcase.assert_close_bf16(dc.out_host(), ref, what=f"wide merge, call {call + 1}")


def test_noalloc_split_minus_one(be):
    cfg = replace(wl.C2, mult_lo=0.5, mult_hi=4.0)
    hc = kvcase.build_case(cfg, batch=4)
    dc = kvcase.DeviceCase(hc)
    ref = _context_entry(be, dc, split=-1)
    dc.out.fill_(0x7FC0)
    assert _noalloc(be, _params(dc, be, split=-1)) == 0
    kvcase.assert_close_bf16(dc.out_host(), ref, what="split -1")
