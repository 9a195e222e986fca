# SPDX-License-Identifier: Apache-2.0
"""GPU parity of the paged decode (through the C ABI) against the oracle.

Tolerance (the parity contract for attention outputs): |gpu - oracle| <=
1e-3 + 2e-2 |oracle| elementwise on the bf16 outputs.
"""
from __future__ import annotations

import ctypes
from dataclasses import replace

import numpy as np
import pytest

import kvcase
from kllm_b200 import Backend, workloads as wl
import kllm_b200 as kb

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    b = Backend()
    assert b.backend == kb.KLLM_GPU_CUDA, "libkllm_gpu found no sm_100 device"
    torch.cuda.set_stream(b.torch_stream())
    yield b
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream())
    b.close()


def run_v2(be, dc, **over):
    import torch
    kw = dc.decode_kwargs(**over)
    kw.setdefault("stream", torch.cuda.current_stream().cuda_stream)
    rc = be.decode_v2(**kw)
    assert rc == 0, f"kllm_gpu_paged_attention_v2 returned {rc}"
    return dc.out_host()


@pytest.mark.parametrize("split", [1, -1])
def test_c1_bf16(be, split):
    hc = kvcase.build_case(wl.C1)
    dc = kvcase.DeviceCase(hc)
    got = run_v2(be, dc, split=split)
    kvcase.assert_close_bf16(got, hc.oracle_decode(), what=f"C1 split={split}")


def test_c2_mx_fp8(be):
    hc = kvcase.build_case(wl.C2, batch=16)
    dc = kvcase.DeviceCase(hc)
    got = run_v2(be, dc)
    kvcase.assert_close_bf16(got, hc.oracle_decode(), what="C2 mx")


@pytest.mark.parametrize("kv", [wl.KV_BF16, wl.KV_MX_FP8])
@pytest.mark.parametrize("block", [32, 64, 128])
def test_block_sizes(be, kv, block):
    cfg = replace(wl.C1, block=block, kv_dtype=kv, arena_slots=None,
                  mult_lo=0.5 if kv else None, mult_hi=4.0 if kv else None)
    hc = kvcase.build_case(cfg, seq_lens=[1, 15, 16, 17, 200, 511, 64, 129])
    dc = kvcase.DeviceCase(hc)
    kvcase.assert_close_bf16(run_v2(be, dc), hc.oracle_decode(), what=f"bs={block} kv={kv}")


@pytest.mark.parametrize("kv", [wl.KV_BF16, wl.KV_MX_FP8])
@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 8), (32, 8), (64, 8), (12, 4)])
def test_gqa_groups(be, kv, hq, hkv):
    cfg = replace(wl.C1, hq=hq, hkv=hkv, kv_dtype=kv, arena_slots=None)
    hc = kvcase.build_case(cfg, seq_lens=[70, 300, 1, 33])
    dc = kvcase.DeviceCase(hc)
    kvcase.assert_close_bf16(run_v2(be, dc), hc.oracle_decode(), what=f"G={hq // hkv}")


@pytest.mark.parametrize("kv", [wl.KV_BF16, wl.KV_MX_FP8])
@pytest.mark.parametrize("hq,hkv", [(16, 4), (4, 4), (8, 4), (32, 4)])
def test_head_dim_64(be, kv, hq, hkv):
    """d = 64 at every merge lane layout (groups 1, 2, 4, 8): short contexts
    are split one tile per warp, so segments of up to 16 tiles are merged by
    the decode itself and longer ones by the wide merge."""
    cfg = replace(wl.C1, d=64, hq=hq, hkv=hkv, kv_dtype=kv, arena_slots=None)
    hc = kvcase.build_case(cfg, seq_lens=[4, 100, 257, 16, 0])
    dc = kvcase.DeviceCase(hc)
    kvcase.assert_close_bf16(run_v2(be, dc), hc.oracle_decode(), what="d=64")


@pytest.mark.parametrize("kv", [wl.KV_BF16, wl.KV_MX_FP8])
def test_edges_empty_invalid_ragged(be, kv):
    """Empty contexts (0 and negative), single tokens, skipped (invalid) pages
    including a skipped last page and a fully skipped sequence."""
    cfg = replace(wl.C1, kv_dtype=kv, arena_slots=None)
    lens = [0, 1, 17, 48, 160, 0, 33, 5, -3, 400]
    invalid = [(2, 0), (3, 2), (4, 3), (4, 4), (6, 2), (7, 0), (9, 10)]
    hc = kvcase.build_case(cfg, seq_lens=lens, invalid=invalid)
    dc = kvcase.DeviceCase(hc)
    dc.out.fill_(0x3F80)  # must be overwritten, zeros included
    got = run_v2(be, dc)
    ref = hc.oracle_decode()
    kvcase.assert_close_bf16(got, ref, what="edges")
    for s in (0, 5, 7, 8):
        assert not got[s].any(), f"seq {s} should be all zeros"


def test_split_equals_whole_long(be):
    """One long context split over every SM vs one warp per segment."""
    cfg = replace(wl.C4, batch=1, ctx_lo=20000, ctx_hi=20000, hq=32)
    hc = kvcase.build_case(cfg)
    dc = kvcase.DeviceCase(hc)
    a = run_v2(be, dc, split=1)
    b = run_v2(be, dc, split=-1)
    ref = hc.oracle_decode()
    kvcase.assert_close_bf16(a, ref, what="split")
    kvcase.assert_close_bf16(b, ref, what="whole")


def test_repeat_calls_counters_reset(be):
    """The split-KV arrival counters must be back at zero after each call."""
    hc = kvcase.build_case(wl.C2, batch=4)
    dc = kvcase.DeviceCase(hc)
    ref = hc.oracle_decode()
    first = run_v2(be, dc)
    for _ in range(3):
        assert np.array_equal(run_v2(be, dc), first)
    kvcase.assert_close_bf16(first, ref, what="repeat")


def test_partials_and_merge(be):
    """partial_m/l/o against the oracle triples; the merge of two halves of a
    context equals the whole-context decode (split-KV across GPUs, on one)."""
    import torch
    cfg = replace(wl.C2, batch=3)
    hc = kvcase.build_case(cfg, seq_lens=[3000, 1, 0])
    dc = kvcase.DeviceCase(hc)
    S, Hq, D = 3, cfg.hq, cfg.d
    pm = torch.empty((S, Hq), dtype=torch.float32, device="cuda")
    pl = torch.empty_like(pm)
    po = torch.empty((S, Hq, D), dtype=torch.float32, device="cuda")
    rc = be.decode_v2(**dc.decode_kwargs(output=None, partial_m=pm.data_ptr(),
                                         partial_l=pl.data_ptr(), partial_o=po.data_ptr()))
    assert rc == 0
    torch.cuda.synchronize()
    m, l, o = hc.oracle_partials()
    kvcase.assert_close_f32(pm.cpu().numpy(), m, atol=2e-3, rtol=1e-3, what="m")
    kvcase.assert_close_f32(pl.cpu().numpy(), l, atol=1e-2, rtol=1e-2, what="l")
    kvcase.assert_close_f32(po.cpu().numpy(), o, what="o")

    # two "ranks": first and second half of every block table
    mb = hc.plan.max_blocks
    half = mb // 2
    lens = hc.seq_lens
    t_all = wl.block_table(hc.plan, cfg, dc.arena.data_ptr(), hc.valid)
    parts = []
    for r in range(2):
        t = np.zeros_like(t_all)
        lo, hi = (0, half) if r == 0 else (half, mb)
        t[:, : hi - lo] = t_all[:, lo:hi]
        l_r = np.clip(lens - lo * cfg.block, 0, (hi - lo) * cfg.block).astype(np.int32)
        tt = torch.from_numpy(t.view(np.uint8).copy()).cuda()
        ll = torch.from_numpy(l_r).cuda()
        m_r = torch.empty((S, Hq), dtype=torch.float32, device="cuda")
        l_rr = torch.empty_like(m_r)
        o_r = torch.empty((S, Hq, D), dtype=torch.float32, device="cuda")
        rc = be.decode_v2(**dc.decode_kwargs(output=None, block_tables=tt.data_ptr(),
                                             seq_lens=ll.data_ptr(), max_blocks_per_seq=mb,
                                             partial_m=m_r.data_ptr(), partial_l=l_rr.data_ptr(),
                                             partial_o=o_r.data_ptr()))
        assert rc == 0
        parts.append((m_r, l_rr, o_r, tt, ll))
    M = torch.stack([p[0] for p in parts]).contiguous()
    L = torch.stack([p[1] for p in parts]).contiguous()
    O = torch.stack([p[2] for p in parts]).contiguous()
    out = torch.zeros((S * Hq, D), dtype=torch.int16, device="cuda")
    rc = be.merge(M.data_ptr(), L.data_ptr(), O.data_ptr(), 2, S * Hq, D, out.data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    merged = out.cpu().numpy().view(np.uint16).reshape(S, Hq, D)
    kvcase.assert_close_bf16(merged, hc.oracle_decode(), what="merge of halves")


def test_v1_entry_points(be):
    """kllm_gpu_paged_attention (ctx) and kllm_gpu_paged_attention_cuda
    (stateless) with the v1 contract: BF16 pages of 128 tokens."""
    import torch
    cfg = replace(wl.C1, block=128, arena_slots=None)
    hc = kvcase.build_case(cfg, seq_lens=[1, 127, 128, 129, 700, 0, 1000, 300])
    dc = kvcase.DeviceCase(hc)
    ref = hc.oracle_decode()
    st = torch.cuda.current_stream().cuda_stream
    rc = be.decode_v1(output=dc.out.data_ptr(), query=dc.q[0].data_ptr(),
                      block_tables=dc.table.data_ptr(), seq_lens=dc.seq_lens.data_ptr(),
                      num_seqs=cfg.batch, num_heads=cfg.hq, num_kv_heads=cfg.hkv,
                      head_dim=cfg.d, max_blocks_per_seq=hc.plan.max_blocks, scale=cfg.scale,
                      stream=st)
    assert rc == 0
    kvcase.assert_close_bf16(dc.out_host(), ref, what="v1 ctx")
    dc.out.zero_()
    rc = be.lib.kllm_gpu_paged_attention_cuda(
        dc.out.data_ptr(), dc.q[0].data_ptr(), dc.table.data_ptr(), dc.seq_lens.data_ptr(),
        cfg.batch, cfg.hq, cfg.hkv, cfg.d, hc.plan.max_blocks, ctypes.c_float(cfg.scale), st)
    assert rc == 0
    kvcase.assert_close_bf16(dc.out_host(), ref, what="v1 stateless")


def test_layers_and_golden_c1(be):
    """Multi-layer pages (layer stride) for layer 1, and C1 against the
    golden output computed by the reference's own code."""
    import golden
    cfg = replace(wl.C2, batch=4, layers=2)
    hc = kvcase.build_case(cfg)
    dc = kvcase.DeviceCase(hc)
    got = run_v2(be, dc, layer=1)
    kvcase.assert_close_bf16(got, hc.oracle_decode(layer=1), what="layer 1")

    hc1 = kvcase.build_case(wl.C1)
    dc1 = kvcase.DeviceCase(hc1)
    kvcase.assert_close_bf16(run_v2(be, dc1), golden.load()["c1_out"], what="C1 golden")


def test_layer_major_arena(be):
    """The same pages laid out layer-major (layer l of every slot in one
    region: slot pitch = one layer's K+V pages, layer stride = n_slots x
    that), decoded for each layer through the ABI's layer stride."""
    import torch
    cfg = replace(wl.C2, batch=5, layers=3)
    hc = kvcase.build_case(cfg, seq_lens=[700, 16, 1, 2049, 333])
    c = hc.cfg
    n = hc.plan.n_slots
    pair = c.layer_stride()
    lm = hc.arena.reshape(n, c.layers, pair).transpose(1, 0, 2).copy()
    dc = kvcase.DeviceCase(hc)
    arena = torch.from_numpy(lm).cuda()
    table = wl.block_table(hc.plan, c, arena.data_ptr(), hc.valid, slot_pitch=pair)
    dc.table = torch.from_numpy(table.view(np.uint8).copy()).cuda()
    for layer in range(c.layers):
        got = run_v2(be, dc, layer=layer, layer_stride=n * pair)
        kvcase.assert_close_bf16(got, hc.oracle_decode(layer=layer), what=f"layer {layer}")


def test_seq_too_long_flag_and_clamp(be):
    import torch
    cfg = replace(wl.C1, arena_slots=None)
    hc = kvcase.build_case(cfg, seq_lens=[64, 64])
    dc = kvcase.DeviceCase(hc)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    dc.seq_lens.copy_(torch.tensor([64, 999], dtype=torch.int32))
    got = run_v2(be, dc, err_word=err.data_ptr())
    assert int(err.item()) & kb.ERR_SEQ_TOO_LONG
    kvcase.assert_close_bf16(got, hc.oracle_decode(), what="clamped")


def test_rejects_bad_shapes(be):
    hc = kvcase.build_case(wl.C1, batch=2)
    dc = kvcase.DeviceCase(hc)
    assert be.decode_v2(**dc.decode_kwargs(head_dim=96)) == kb.ENOSYS
    assert be.decode_v2(**dc.decode_kwargs(num_heads=30)) == kb.EINVAL
    assert be.decode_v2(**dc.decode_kwargs(block_size=24)) == kb.ENOSYS
    assert be.decode_v2(**dc.decode_kwargs(kv_dtype=7)) == kb.ENOSYS
    assert be.decode_v2(**dc.decode_kwargs(layer_stride=8)) == kb.EINVAL
    assert be.decode_v2(**dc.decode_kwargs(layer=-1)) == kb.EINVAL


def test_c4_long_context_wide_merge(be):
    """C4 at full size: one 131072-token context, 64 q / 8 kv heads. Every kv
    head is split over hundreds of warps, so the partials go through the
    queued wide merge; bf16 output and partial triples against the oracle."""
    import torch
    hc = kvcase.build_case(wl.C4)
    dc = kvcase.DeviceCase(hc)
    ref = hc.oracle_decode()
    kvcase.assert_close_bf16(run_v2(be, dc), ref, what="C4")
    c = hc.cfg
    pm = torch.empty((1, c.hq), dtype=torch.float32, device="cuda")
    pl = torch.empty_like(pm)
    po = torch.empty((1, c.hq, c.d), dtype=torch.float32, device="cuda")
    rc = be.decode_v2(**dc.decode_kwargs(output=None, partial_m=pm.data_ptr(),
                                         partial_l=pl.data_ptr(), partial_o=po.data_ptr()))
    assert rc == 0
    torch.cuda.synchronize()
    m, l, o = hc.oracle_partials()
    kvcase.assert_close_f32(pm.cpu().numpy(), m, atol=2e-3, rtol=1e-3, what="m")
    kvcase.assert_close_f32(pl.cpu().numpy(), l, atol=1e-2, rtol=1e-2, what="l")
    kvcase.assert_close_f32(po.cpu().numpy(), o, what="o")
    # a second call finds the merge queue empty again
    kvcase.assert_close_bf16(run_v2(be, dc), ref, what="C4 again")


def test_overlap_flag_layers_and_append(be):
    """KLLM_DECODE_OVERLAP_PREV: each decode may start while the kernel before
    it finishes. Three layers decoded back to back into separate outputs, and
    a decode issued right after a KV append that rewrites the last token of
    every sequence: the decode must see the appended bytes (it reads pages
    only after the previous kernel completed)."""
    import torch
    cfg = replace(wl.C2, batch=6, layers=3)
    hc = kvcase.build_case(cfg, seq_lens=[700, 16, 1, 2049, 333, 4096])
    c = hc.cfg
    dc = kvcase.DeviceCase(hc)
    st = torch.cuda.current_stream().cuda_stream
    outs = [torch.zeros_like(dc.out) for _ in range(c.layers)]
    for layer in range(c.layers):
        rc = be.decode_v2(**dc.decode_kwargs(layer=layer, output=outs[layer].data_ptr(),
                                             flags=kb.DECODE_OVERLAP_PREV, stream=st))
        assert rc == 0
    torch.cuda.synchronize()
    for layer in range(c.layers):
        got = outs[layer].cpu().numpy().view(np.uint16)
        kvcase.assert_close_bf16(got, hc.oracle_decode(layer=layer), what=f"layer {layer}")

    # append -> decode (layer 1), the decode launched as a dependent of the append
    import oracle
    S = c.batch
    tok_seq = np.arange(S, dtype=np.int32)
    tok_pos = (hc.seq_lens - 1).astype(np.int32)
    k = wl.normal_bf16(5, wl.ST_PK, 0, (S, c.hkv, c.d), mult=3.0)
    v = wl.normal_bf16(5, wl.ST_PV, 0, (S, c.hkv, c.d), mult=3.0)
    tk = torch.from_numpy(k.view(np.int16)).cuda()
    tv = torch.from_numpy(v.view(np.int16)).cuda()
    ts = torch.from_numpy(tok_seq).cuda()
    tp = torch.from_numpy(tok_pos).cuda()
    rc = be.append(k=tk.data_ptr(), v=tv.data_ptr(), token_seq=ts.data_ptr(),
                   token_pos=tp.data_ptr(), num_tokens=S, num_seqs=S,
                   block_tables=dc.table.data_ptr(), max_blocks_per_seq=hc.plan.max_blocks,
                   num_kv_heads=c.hkv, head_dim=c.d, block_size=c.block, kv_dtype=c.kv_dtype,
                   layer=1, layer_stride=c.layer_stride(), stream=st)
    assert rc == 0
    dc.out.fill_(0x7FC0)
    rc = be.decode_v2(**dc.decode_kwargs(layer=1, flags=kb.DECODE_OVERLAP_PREV, stream=st))
    assert rc == 0
    got = dc.out_host()
    n = oracle.kv_append(k, v, tok_seq, tok_pos, hc.host_table(), hc.plan.max_blocks, c.hkv,
                         c.d, c.block, c.kv_dtype, hc.layer_off(1))
    assert n == 0, f"oracle append skipped {n} rows"
    kvcase.assert_close_bf16(got, hc.oracle_decode(layer=1), what="decode after append")
    # unknown flag bits are refused
    assert be.decode_v2(**dc.decode_kwargs(flags=0x2)) == kb.EINVAL


@pytest.mark.parametrize("split", [1, -1])
def test_mx_decode_every_payload_code(be, split):
    """Every E4M3 payload code through the decode kernel, 0x7F / 0xFF
    included (the reference decodes them as +-480, the hardware conversion
    as NaN: such pieces are recomputed exactly). Payload bytes of every K
    and V page are overwritten with a pattern that cycles through all 256
    codes; the scale bytes stay the quantizer's. One long context is split
    over many warps (partials and merges), the others are short."""
    cfg = replace(wl.C2, batch=4)
    hc = kvcase.build_case(cfg, seq_lens=[5000, 37, 700, 16])
    c = hc.cfg
    sec, pay = c.section_bytes(), c.block * c.d
    t = np.arange(c.block)[:, None]
    d = np.arange(c.d)[None, :]
    for s_, L in enumerate(hc.seq_lens):
        n_pages = (int(L) + c.block - 1) // c.block
        for b in range(n_pages):
            slot = hc.plan.slots[s_, b]
            for which in range(2):
                for h in range(c.hkv):
                    pat = ((t * 131 + d * 7 + h * 31 + b * 13 + which * 101 + s_ * 59)
                           % 256).astype(np.uint8)
                    off = which * c.page_bytes() + h * sec
                    hc.arena[slot, off:off + pay] = pat.reshape(-1)
    codes = set()
    for h in range(c.hkv):
        codes |= set(np.unique(hc.arena[hc.plan.slots[0, 0], h * sec:h * sec + pay]).tolist())
    assert codes == set(range(256))
    dc = kvcase.DeviceCase(hc)
    dc.out.fill_(0x7FC0)
    got = run_v2(be, dc, split=split)
    kvcase.assert_close_bf16(got, hc.oracle_decode(), what=f"all payload codes, split={split}")


def test_registered_arenas_page_range_checks(be):
    """With arenas registered, a page outside all of them is skipped by the
    decode (KLLM_ERR_PAGE_RANGE, output as if the entry were invalid) and
    never written by the append."""
    import torch
    cfg = replace(wl.C2, batch=5)
    hc = kvcase.build_case(cfg, seq_lens=[700, 16, 1, 2049, 333])
    c = hc.cfg
    dc = kvcase.DeviceCase(hc)
    lib, ctx = be.lib, be.ctx
    n = hc.plan.n_slots
    slot_b = c.slot_bytes()
    base = dc.arena.data_ptr()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    try:
        # the whole arena registered: nothing changes
        assert lib.kllm_gpu_register_arena(ctx, base, n * slot_b) == 0
        got = run_v2(be, dc, err_word=err.data_ptr())
        assert int(err.item()) == 0
        kvcase.assert_close_bf16(got, hc.oracle_decode(), what="whole arena registered")
        # only the first half of the slots registered
        lib.kllm_gpu_clear_arenas(ctx)
        half = n // 2
        assert lib.kllm_gpu_register_arena(ctx, base, half * slot_b) == 0
        got = run_v2(be, dc, err_word=err.data_ptr())
        assert int(err.item()) & kb.ERR_PAGE_RANGE
        ref_case = replace(hc, valid=hc.valid & (hc.plan.slots < half))
        kvcase.assert_close_bf16(got, ref_case.oracle_decode(), what="half the arena registered")
        # an append into an unregistered page leaves it untouched
        before = dc.arena.clone()
        s_out = int(np.argwhere(hc.plan.slots[0] >= half)[0][0]) if (hc.plan.slots[0] >= half).any() \
            else None
        if s_out is not None:
            err.zero_()
            kk = torch.zeros((1, c.hkv, c.d), dtype=torch.int16, device="cuda").fill_(0x3F80)
            ts = torch.zeros(1, dtype=torch.int32, device="cuda")
            tp = torch.full((1,), s_out * c.block, dtype=torch.int32, device="cuda")
            rc = be.append(k=kk.data_ptr(), v=kk.data_ptr(), token_seq=ts.data_ptr(),
                           token_pos=tp.data_ptr(), num_tokens=1, num_seqs=c.batch,
                           block_tables=dc.table.data_ptr(), max_blocks_per_seq=hc.plan.max_blocks,
                           num_kv_heads=c.hkv, head_dim=c.d, block_size=c.block,
                           kv_dtype=c.kv_dtype, layer=0, layer_stride=c.layer_stride(),
                           err_word=err.data_ptr(), stream=torch.cuda.current_stream().cuda_stream)
            assert rc == 0
            torch.cuda.synchronize()
            assert int(err.item()) & kb.ERR_PAGE_RANGE
            assert torch.equal(before, dc.arena), "an unregistered page was written"
    finally:
        lib.kllm_gpu_clear_arenas(ctx)


def test_trace_records(be):
    """Per-call GPU timing: one record per traced call, in call order, with
    the caller's tag, the host submit time and the device time."""
    import ctypes as ct
    import torch
    lib, ctx = be.lib, be.ctx
    hc = kvcase.build_case(wl.C2, batch=8)
    dc = kvcase.DeviceCase(hc)
    assert lib.kllm_gpu_trace_enable(ctx, 4) == 0
    try:
        lib.kllm_gpu_trace_tag(ctx, 77)
        for _ in range(6):     # two beyond the ring's capacity: dropped
            be.decode_v2(**dc.decode_kwargs(
                stream=torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        recs = (kb.TraceRecord * 8)()
        dropped = ct.c_uint64(0)
        n = lib.kllm_gpu_trace_read(ctx, recs, 8, ct.byref(dropped))
        assert n == 4 and dropped.value == 2
        assert [recs[i].op for i in range(n)] == [kb.TRACE_DECODE] * 4
        assert all(recs[i].tag == 77 and recs[i].gpu_us > 0 for i in range(n))
        assert [recs[i].seq for i in range(n)] == [0, 1, 2, 3]
        assert all(recs[i + 1].submit_ns >= recs[i].submit_ns for i in range(n - 1))
        # the ring has room again
        be.decode_v2(**dc.decode_kwargs(stream=torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert lib.kllm_gpu_trace_read(ctx, recs, 8, None) == 1 and recs[0].seq == 4
    finally:
        assert lib.kllm_gpu_trace_enable(ctx, 0) == 0
