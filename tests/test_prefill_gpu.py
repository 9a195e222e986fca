# SPDX-License-Identifier: Apache-2.0
"""GPU parity of chunked prefill (tcgen05) through the C ABI.

Row j of sequence s's chunk attends to the sequence's cached context
(positions 0..ctx-1, read from the paged cache) and chunk keys 0..j; the
oracle computes the same rows with orc_attention over the gathered keys
(the reference CPU attention applied per row). Tolerance: 1e-3 + 2e-2 |ref|.
With append = 1 the chunk's K/V land in the cache bit-exactly as the oracle
quantizer writes them."""
from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest

import kvcase
import oracle
import kllm_b200 as kb
from kllm_b200 import Backend, workloads as wl

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    import torch
    assert torch.cuda.is_available()
    b = Backend()
    assert b.backend == kb.KLLM_GPU_CUDA
    torch.cuda.set_stream(b.torch_stream())
    yield b
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream())
    b.close()


def _case(cfg, ctx_lens, chunk_lens, seed=5, invalid=None, share_prefix=0):
    """Cache holding ctx + chunk tokens per sequence (the chunk part gets
    overwritten by the append); chunk Q/K/V packed token-major."""
    ctx_lens = np.asarray(ctx_lens, np.int32)
    chunk_lens = np.asarray(chunk_lens, np.int32)
    total = ctx_lens + chunk_lens
    hc = kvcase.build_case(cfg, seq_lens=total, invalid=invalid, seed=seed)
    if share_prefix:  # sequences 1.. reuse sequence 0's first pages (cache hits)
        npg = share_prefix // cfg.block
        for s in range(1, len(total)):
            if ctx_lens[s] >= share_prefix:
                hc.plan.slots[s, :npg] = hc.plan.slots[0, :npg]
    n = int(chunk_lens.sum())
    cu = np.concatenate([[0], np.cumsum(chunk_lens)]).astype(np.int32)
    q = wl.normal_bf16(seed, wl.ST_PQ, 0, (n, cfg.hq, cfg.d))
    k = wl.normal_bf16(seed, wl.ST_PK, 0, (n, cfg.hkv, cfg.d))
    v = wl.normal_bf16(seed, wl.ST_PV, 0, (n, cfg.hkv, cfg.d))
    return hc, ctx_lens, chunk_lens, cu, q, k, v


def _oracle_rows(hc, ctx_lens, cu, q, k, v, rows=None):
    """Expected output rows [n, hq, d] (rows: optional subset of token rows)."""
    c = hc.cfg
    g = c.hq // c.hkv
    table = hc.host_table()
    out = {}
    for s in range(len(ctx_lens)):
        a, b = int(cu[s]), int(cu[s + 1])
        want = range(a, b) if rows is None else [r for r in rows if a <= r < b]
        if not want:
            continue
        for h in range(c.hkv):
            kp, vp = oracle.gather(table[s], hc.plan.max_blocks, int(ctx_lens[s]), h, c.hkv,
                                   c.d, c.block, c.kv_dtype)
            kall = np.concatenate([kp, k[a:b, h]], axis=0)
            vall = np.concatenate([vp, v[a:b, h]], axis=0)
            for r in want:
                j = r - a
                n_keys = len(kp) + j + 1
                qg = q[r, h * g:(h + 1) * g][:, None, :]
                o = oracle.attention(qg, kall[:n_keys, None], vall[:n_keys, None], 1, c.d,
                                     n_keys, g, c.scale)
                out.setdefault(r, np.zeros((c.hq, c.d), np.uint16))[h * g:(h + 1) * g] = o[:, 0]
    return out


def _run(be, hc, ctx_lens, chunk_lens, cu, q, k, v, append=1):
    import torch
    dc = kvcase.DeviceCase(hc)
    c = hc.cfg
    if hasattr(hc, "_shared"):
        pass
    table = wl.block_table(hc.plan, c, dc.arena.data_ptr(), hc.valid)
    dc.table = torch.from_numpy(table.view(np.uint8).copy()).cuda()
    td = {n: torch.from_numpy(x.view(np.int16).copy() if x.dtype == np.uint16 else x.copy()).cuda()
          for n, x in (("q", q), ("k", k), ("v", v), ("cu", cu), ("ctx", ctx_lens))}
    out = torch.full((len(q), c.hq, c.d), 0x7FC0, dtype=torch.int16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = be.prefill(output=out.data_ptr(), q=td["q"].data_ptr(), k=td["k"].data_ptr(),
                    v=td["v"].data_ptr(), cu_seqlens=td["cu"].data_ptr(),
                    ctx_lens=td["ctx"].data_ptr(), num_seqs=len(ctx_lens), num_tokens=len(q),
                    max_chunk=int(chunk_lens.max()), num_heads=c.hq, num_kv_heads=c.hkv,
                    head_dim=c.d, block_tables=dc.table.data_ptr(),
                    max_blocks_per_seq=hc.plan.max_blocks, block_size=c.block,
                    kv_dtype=c.kv_dtype, layer=0, layer_stride=c.layer_stride(), scale=c.scale,
                    append=append, err_word=err.data_ptr(),
                    stream=torch.cuda.current_stream().cuda_stream)
    assert rc == 0, (rc, "cuda error", be.stats().last_cuda_error)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, hex(int(err.item()))
    return out.cpu().numpy().view(np.uint16), dc.arena.cpu().numpy()


def _check(got, want, what):
    for r, w in want.items():
        kvcase.assert_close_bf16(got[r], w, what=f"{what} row {r}")


@pytest.mark.parametrize("kv", [wl.KV_MX_FP8, wl.KV_BF16])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (16, 16), (64, 8), (16, 8)])
def test_prefill_small(be, kv, hq, hkv):
    cfg = replace(wl.C2, kv_dtype=kv, hq=hq, hkv=hkv, mult_lo=None, mult_hi=None)
    case = _case(cfg, ctx_lens=[0, 37, 300, 128], chunk_lens=[200, 70, 33, 129])
    hc, ctx_lens, chunk_lens, cu, q, k, v = case
    want = _oracle_rows(hc, ctx_lens, cu, q, k, v)
    got, _ = _run(be, *case)
    _check(got, want, f"kv={kv} g={hq // hkv}")


def test_prefill_invalid_prior_page_and_append_bit_exact(be):
    cfg = replace(wl.C2, mult_lo=None, mult_hi=None)
    case = _case(cfg, ctx_lens=[160, 64], chunk_lens=[100, 50], invalid=[(0, 3)])
    hc, ctx_lens, chunk_lens, cu, q, k, v = case
    want = _oracle_rows(hc, ctx_lens, cu, q, k, v)
    got, arena = _run(be, *case)
    _check(got, want, "invalid page")
    # the oracle appends the chunk into the host arena the same way
    tok_seq = np.repeat(np.arange(len(ctx_lens)), chunk_lens).astype(np.int32)
    tok_pos = np.concatenate([np.arange(c0, c0 + n) for c0, n in zip(ctx_lens, chunk_lens)])
    oracle.kv_append(k, v, tok_seq, tok_pos.astype(np.int32), hc.host_table(),
                     hc.plan.max_blocks, cfg.hkv, cfg.d, cfg.block, cfg.kv_dtype)
    assert np.array_equal(arena, hc.arena), "append differs from the oracle"


def test_prefill_c5_shared_prefix_sampled(be):
    """C5 shape: 16 prompts of 2048 tokens, 32q/8kv; 4 of them hit a shared
    1024-token prefix chain in the MX cache and prefill only their last 1024
    tokens. Rows are sampled for the oracle (it is O(L^2) per row)."""
    cfg = replace(wl.C2, mult_lo=None, mult_hi=None)
    ctx = [1024] * 4 + [0] * 12
    chunk = [1024] * 4 + [2048] * 12
    case = _case(cfg, ctx_lens=ctx, chunk_lens=chunk, share_prefix=1024)
    hc, ctx_lens, chunk_lens, cu, q, k, v = case
    # the shared prefix pages hold sequence 0's prefix for all four
    rng = np.random.default_rng(0)
    rows = sorted(set(rng.integers(0, int(cu[-1]), 48).tolist()) |
                  {0, int(cu[1]) - 1, int(cu[4]), int(cu[4]) + 127, int(cu[-1]) - 1})
    want = _oracle_rows(hc, ctx_lens, cu, q, k, v, rows=rows)
    got, arena = _run(be, *case)
    _check(got, want, "C5")
    # the chunk's 28,672 tokens appended on write, byte for byte
    tok_seq = np.repeat(np.arange(len(ctx_lens)), chunk_lens).astype(np.int32)
    tok_pos = np.concatenate([np.arange(c0, c0 + n) for c0, n in zip(ctx_lens, chunk_lens)])
    oracle.kv_append(k, v, tok_seq, tok_pos.astype(np.int32), hc.host_table(),
                     hc.plan.max_blocks, cfg.hkv, cfg.d, cfg.block, cfg.kv_dtype)
    assert np.array_equal(arena, hc.arena), "C5 append differs from the oracle"


@pytest.mark.parametrize("kv", [wl.KV_MX_FP8, wl.KV_BF16])
@pytest.mark.parametrize("block", [32, 128])
def test_prefill_edges(be, kv, block):
    """An empty chunk, one-token chunks over short and empty contexts, a
    context that ends one past a page, chunks that cross tile boundaries;
    pages of 32 and 128 tokens; K/V magnitudes scaled per (sequence, head)
    by 0.5 .. 4 as in the C2 workload."""
    cfg = replace(wl.C2, kv_dtype=kv, block=block)
    case = _case(cfg, ctx_lens=[5, 0, 257, 31, 1, 0], chunk_lens=[1, 0, 65, 300, 128, 1],
                 seed=9)
    hc, ctx_lens, chunk_lens, cu, q, k, v = case
    want = _oracle_rows(hc, ctx_lens, cu, q, k, v)
    got, _ = _run(be, *case)
    _check(got, want, f"edges kv={kv} block={block}")
