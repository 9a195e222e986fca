# SPDX-License-Identifier: Apache-2.0
"""kllm_gpu_paged_attention_v2_noalloc: the decode entry point for callers
that may not allocate device memory (for instance a polling reactor thread
under a zero-allocation rule, where cudaMalloc can stall or fail once the KV
arena owns the GPU). It keeps its split-KV scratch in a fixed array inside
the library instead of a context workspace.

Checked through the C ABI against kllm_gpu_paged_attention_v2 on two calls in
a row (the second call runs on scratch the first one left behind), with the
same tolerance as the other parity tests. This file is collected last so
that a run stopping at its first failure has run every other test first.
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


@pytest.mark.parametrize("kv", [wl.KV_MX_FP8, wl.KV_BF16])
def test_noalloc_matches_context_entry_point_twice(kv):
    import torch
    assert torch.cuda.is_available()
    lib = kb.load()
    be = kb.Backend(lib)
    assert be.backend == kb.KLLM_GPU_CUDA
    torch.cuda.set_stream(be.torch_stream())
    try:
        cfg = replace(wl.C2, kv_dtype=kv, mult_lo=0.5, mult_hi=4.0)
        hc = kvcase.build_case(cfg, batch=8)
        dc = kvcase.DeviceCase(hc)
        st = be.stream
        assert be.decode_v2(**dc.decode_kwargs(stream=st)) == 0
        ref = dc.out_host().copy()
        kvcase.assert_close_bf16(ref, hc.oracle_decode(), what="context entry point")

        outs = []
        for _ in range(2):
            dc.out.fill_(0x7FC0)   # NaN: every element must be written
            p = kb.AttnParamsV2()
            p.struct_size = ctypes.sizeof(p)
            for k, v in dc.decode_kwargs(stream=st).items():
                setattr(p, k, v)
            assert lib.kllm_gpu_paged_attention_v2_noalloc(ctypes.byref(p)) == 0
            outs.append(dc.out_host().copy())
        for i, got in enumerate(outs):
            kvcase.assert_close_bf16(got, ref, what=f"no-alloc call {i + 1}")
        assert np.array_equal(outs[0], outs[1]), "second call differs from the first"

        # sizes beyond the scratch's counter capacity are refused up front
        p = kb.AttnParamsV2()
        p.struct_size = ctypes.sizeof(p)
        for k, v in dc.decode_kwargs(stream=st).items():
            setattr(p, k, v)
        p.num_seqs = 65536 // cfg.hkv + 1
        assert lib.kllm_gpu_paged_attention_v2_noalloc(ctypes.byref(p)) == kb.ENOSPC
    finally:
        torch.cuda.synchronize()
        torch.cuda.set_stream(torch.cuda.default_stream())
        be.close()
