# SPDX-License-Identifier: Apache-2.0
"""GPU parity of the cache-side kernels through the C ABI: quantize-on-write
append (bit-exact), the logical gather (bit-exact), the partial merge."""
from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest

import kvcase
import oracle
from kllm_b200 import Backend, workloads as wl
import kllm_b200 as kb

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


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def _random_bits_bf16(shape, seed):
    """bf16 values with random signs and mantissas over 2^-20 .. 2^18 (38
    binades, so every E4M3 scale code and many exact-midpoint quotients occur),
    one in 16 zero."""
    rng = np.random.default_rng(seed)
    exp = rng.integers(107, 145, size=shape, dtype=np.uint16)
    bits = (rng.integers(0, 2, size=shape, dtype=np.uint16) << 15) | (exp << 7) | \
        rng.integers(0, 128, size=shape, dtype=np.uint16)
    bits[rng.integers(0, 16, size=shape) == 0] = 0
    return bits.astype(np.uint16)


# micro-blocks with infinities and NaNs (bf16 bits): an infinity among
# finite values, a NaN among finite values, infinities only, NaNs only (both
# signs, quiet and signalling: abs-max 0, so the block is zero), NaN with
# infinity, and a NaN beside values that quantize to subnormal codes
_NONFINITE_BLOCKS = [
    [0x7F80, 0x3F80, 0x4000, 0x4040, 0xC080, 0x40A0, 0x40C0, 0x40E0],
    [0x7FC0, 0x3F80, 0xC000, 0x3F00, 0x0000, 0x8000, 0x0000, 0x3F80],
    [0xFF80, 0xFF80, 0x7F80, 0x0000, 0x0000, 0x0000, 0x0000, 0x0000],
    [0x7FC0, 0xFFC0, 0x7F81, 0xFF81, 0x7FC0, 0x7FC0, 0xFFC0, 0x7FFF],
    [0x7FC0, 0x7F80, 0xFFC0, 0x4040, 0x0000, 0xC040, 0x0000, 0x3F80],
    [0xFFC0, 0x3C00, 0xBC00, 0x3B80, 0x0000, 0x3A00, 0x0000, 0x3C80],
]


def _append_case(kv, block=16, d=128, hkv=8, seed=3, n_seq=5, extreme=False,
                 random_bits=False, nonfinite=False, lens=None):
    """Random tokens appended at scattered positions of a few sequences."""
    cfg = replace(wl.C1, kv_dtype=kv if kv != 2 else wl.KV_BF16, block=block, d=d, hkv=hkv,
                  hq=hkv, arena_slots=None)
    lens = np.array([33, 70, 16, 1, 129][:n_seq] if lens is None else lens, dtype=np.int32)
    plan = wl.plan_pages(cfg, lens, seed)
    pos = np.concatenate([np.arange(L) for L in lens]).astype(np.int32)
    seq = np.concatenate([np.full(L, s) for s, L in enumerate(lens)]).astype(np.int32)
    perm = wl.permutation(len(pos), seed, 7)
    pos, seq = pos[perm], seq[perm]
    n = len(pos)
    k = wl.normal_bf16(seed, wl.ST_PK, 0, (n, hkv, d))
    v = wl.normal_bf16(seed, wl.ST_PV, 0, (n, hkv, d))
    if random_bits:
        k = _random_bits_bf16((n, hkv, d), seed)
        v = _random_bits_bf16((n, hkv, d), seed + 1)
    if extreme:  # zeros, huge, tiny, subnormal-producing blocks, signed zeros
        kf = wl.bf16_to_f32(k).copy()
        kf[0, 0, :8] = 0.0
        kf[1, 0, :8] = np.array([3e5, -2e5, 1, 0, 5, 7, -1e5, 2e4])
        kf[2, 0, :8] = np.array([1e-30, -2e-31, 3e-32, 0, 1e-33, 4e-30, -1e-30, 2e-30])
        kf[3, 0, :8] = np.array([448, -448, 447, 449, 0.001, -0.002, 464, 480])
        kf[4, 0, :8] = -0.0
        kf[5, 0, :8] = np.array([1.0, 1 / 64, 1 / 512, 1 / 1024, 1 / 700, 3 / 1024, 0, -1])
        kf[6, 0, :8] = np.array([-0.0, 1, -0.0, 2, 0, -3, -0.0, 4])  # signed zeros kept
        k = wl.f32_to_bf16(kf)
    if nonfinite:
        k, v = k.copy(), v.copy()
        for t, blk in enumerate(_NONFINITE_BLOCKS):
            k[t, 0, :8] = blk
            v[t + 1, hkv - 1, d - 8:] = blk
    return cfg, plan, seq, pos, k, v


def _section_bytes(kv, block, d):
    if kv == wl.KV_MX_FP8:
        return block * d + block * d // 8
    if kv == 2:
        return block * d * 2 + block * d // 8
    return block * d * 2


@pytest.mark.parametrize("kv", [wl.KV_BF16, wl.KV_MX_FP8, 2])
@pytest.mark.parametrize("extreme", [False, True])
def test_append_bit_exact(be, kv, extreme, random_bits=False, block=16, d=128, hkv=8,
                          offset=0, nonfinite=False, lens=None):
    import torch
    cfg, plan, seq, pos, k, v = _append_case(kv, extreme=extreme, random_bits=random_bits,
                                             block=block, d=d, hkv=hkv, nonfinite=nonfinite,
                                             lens=lens)
    sec = _section_bytes(kv, cfg.block, cfg.d)
    page = cfg.hkv * sec
    slot_bytes = 2 * page
    arena_h = np.zeros((plan.n_slots, slot_bytes + offset), dtype=np.uint8)
    arena_d = torch.zeros((plan.n_slots, slot_bytes + offset), dtype=torch.uint8,
                          device="cuda")
    slot_bytes += offset   # pages offset within 16-byte alignment when offset % 16 != 0

    def table(base):
        t = np.zeros(plan.slots.shape, dtype=wl.ENTRY_DTYPE)
        used = plan.slots >= 0
        addr = np.uint64(base + offset) + plan.slots.clip(0).astype(np.uint64) * \
            np.uint64(slot_bytes)
        t["k"] = np.where(used, addr, 0)
        t["v"] = np.where(used, addr + np.uint64(page), 0)
        t["valid"] = used
        return t

    skipped = oracle.kv_append(k, v, seq, pos, table(arena_h.ctypes.data), plan.max_blocks,
                               cfg.hkv, cfg.d, cfg.block, kv)
    assert skipped == 0
    td = torch.from_numpy(table(arena_d.data_ptr()).view(np.uint8).copy()).cuda()
    kd = torch.from_numpy(k.view(np.int16).copy()).cuda()
    vd = torch.from_numpy(v.view(np.int16).copy()).cuda()
    sd = torch.from_numpy(seq).cuda()
    pd = torch.from_numpy(pos).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = be.append(k=kd.data_ptr(), v=vd.data_ptr(), token_seq=sd.data_ptr(),
                   token_pos=pd.data_ptr(), num_tokens=len(seq), num_seqs=len(plan.seq_lens),
                   block_tables=td.data_ptr(),
                   max_blocks_per_seq=plan.max_blocks, num_kv_heads=cfg.hkv, head_dim=cfg.d,
                   block_size=cfg.block, kv_dtype=kv, err_word=err.data_ptr(),
                   stream=_stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = arena_d.cpu().numpy()
    if not np.array_equal(got, arena_h):
        diff = np.argwhere(got != arena_h)
        raise AssertionError(f"{len(diff)} bytes differ; first {diff[:5].tolist()}")


@pytest.mark.parametrize("kv", [wl.KV_BF16, wl.KV_MX_FP8])
@pytest.mark.parametrize("block,d,hkv", [(32, 64, 4), (16, 128, 16), (64, 64, 1), (128, 128, 2)])
def test_append_shapes_bit_exact(be, kv, block, d, hkv):
    """Head dims 64 and 128 with 1 to 16 kv heads (16 x 128: more than one
    pass of the warp over a token's row) and blocks of 16 to 128 tokens."""
    test_append_bit_exact(be, kv, True, random_bits=kv == wl.KV_MX_FP8, block=block, d=d,
                          hkv=hkv)


@pytest.mark.parametrize("d", [128, 64, 32])
def test_append_nonfinite_bit_exact(be, d):
    """Infinities and NaNs in K and V (head dims 128 and 64: the warp kernel;
    32: the general kernel) are quantized as the oracle does: NaNs left out
    of the abs-max, an infinite abs-max saturating the scale at 0x7E, NaN
    and infinite elements encoded as S.1111.111 and S.1111.110."""
    test_append_bit_exact(be, wl.KV_MX_FP8, False, random_bits=True, d=d, nonfinite=True)


@pytest.mark.parametrize("kv", [wl.KV_BF16, wl.KV_MX_FP8])
def test_append_many_tokens_bit_exact(be, kv):
    """More tokens (24,576, scattered over 12 sequences) than the grid has
    warps, so each warp quantizes several."""
    test_append_bit_exact(be, kv, True, random_bits=kv == wl.KV_MX_FP8, nonfinite=True,
                          lens=[4096, 1, 2047, 3000, 17, 4500, 2048, 2049, 600, 3000, 1200, 2018])


def test_append_pages_8_byte_aligned(be):
    """MX pages only 8-byte aligned: scale bytes are written one by one
    instead of as a 16-byte row, with the same result."""
    test_append_bit_exact(be, wl.KV_MX_FP8, False, random_bits=True, offset=8)


@pytest.mark.parametrize("kv", [wl.KV_MX_FP8, 2])
def test_append_random_bits_bit_exact(be, kv):
    """Quantize-on-write of random bf16 bit patterns over 38 binades: the
    GPU's reciprocal-and-residual quotient must round to the same E4M3 codes
    as the oracle's exact division, ties included."""
    test_append_bit_exact(be, kv, False, random_bits=True)


def test_append_compat_matches_reference_function(be):
    """kv_dtype 2 reproduces the reference's mx_quant_to_bf16 bit for bit
    (checked here against the oracle restatement, itself pinned to the
    reference by tests/test_oracle.py)."""
    test_append_bit_exact(be, 2, True)


def test_append_missing_page_flag(be):
    import torch
    cfg, plan, seq, pos, k, v = _append_case(wl.KV_MX_FP8)
    t = np.zeros(plan.slots.shape, dtype=wl.ENTRY_DTYPE)   # every entry invalid
    td = torch.from_numpy(t.view(np.uint8).copy()).cuda()
    kd = torch.from_numpy(k.view(np.int16).copy()).cuda()
    sd = torch.from_numpy(seq).cuda()
    pd = torch.from_numpy(pos).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = be.append(k=kd.data_ptr(), v=kd.data_ptr(), token_seq=sd.data_ptr(),
                   token_pos=pd.data_ptr(), num_tokens=len(seq), num_seqs=len(plan.seq_lens),
                   block_tables=td.data_ptr(),
                   max_blocks_per_seq=plan.max_blocks, num_kv_heads=cfg.hkv, head_dim=cfg.d,
                   block_size=cfg.block, kv_dtype=1, err_word=err.data_ptr(), stream=_stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) & kb.ERR_APPEND_NOPAGE


def _gather_check(be, hc):
    import torch
    dc = kvcase.DeviceCase(hc)
    c = hc.cfg
    cap = hc.plan.max_blocks * c.block
    ko = torch.zeros((c.batch, c.hkv, cap, c.d), dtype=torch.int16, device="cuda")
    vo = torch.zeros_like(ko)
    cnt = torch.zeros((c.batch, c.hkv), dtype=torch.int32, device="cuda")
    rc = be.gather(k_out=ko.data_ptr(), v_out=vo.data_ptr(), counts_out=cnt.data_ptr(),
                   block_tables=dc.table.data_ptr(), seq_lens=dc.seq_lens.data_ptr(),
                   num_seqs=c.batch, num_kv_heads=c.hkv, head_dim=c.d,
                   max_blocks_per_seq=hc.plan.max_blocks, block_size=c.block,
                   kv_dtype=c.kv_dtype, stream=_stream())
    assert rc == 0
    torch.cuda.synchronize()
    ko = ko.cpu().numpy().view(np.uint16)
    vo = vo.cpu().numpy().view(np.uint16)
    cnt = cnt.cpu().numpy()
    table = hc.host_table()
    for s in range(c.batch):
        for h in range(c.hkv):
            rk, rv = oracle.gather(table[s], hc.plan.max_blocks, int(hc.seq_lens[s]), h, c.hkv,
                                   c.d, c.block, c.kv_dtype)
            n = len(rk)
            assert cnt[s, h] == n
            assert np.array_equal(ko[s, h, :n], rk), (s, h)
            assert np.array_equal(vo[s, h, :n], rv), (s, h)
            assert not ko[s, h, n:].any() and not vo[s, h, n:].any()


@pytest.mark.parametrize("kv", [wl.KV_BF16, wl.KV_MX_FP8])
def test_gather_bit_exact(be, kv):
    cfg = replace(wl.C1, kv_dtype=kv, arena_slots=None)
    hc = kvcase.build_case(cfg, seq_lens=[1, 17, 300, 0, 64, 95],
                           invalid=[(1, 0), (2, 5), (5, 5)])
    _gather_check(be, hc)


def test_gather_every_e4m3_code(be):
    """Every payload code under every scale code dequantises exactly as the
    reference decoder (userspace/compute/mx_dequant.h:30-55) says."""
    cfg = replace(wl.C1, kv_dtype=wl.KV_MX_FP8, hkv=1, hq=1, arena_slots=None)
    hc = kvcase.build_case(cfg, seq_lens=[512])   # 512 tokens x 16 scale blocks
    sec = cfg.section_bytes()
    codes = np.arange(256, dtype=np.uint8)
    for b in range(hc.plan.max_blocks):
        slot = hc.plan.slots[0, b]
        for which in (0, 1):
            base = which * cfg.page_bytes()
            pay = np.tile(codes, cfg.block * cfg.d // 256)
            sc_codes = (np.arange(cfg.block * cfg.d // 8) + b * 7 + which) % 256
            hc.arena[slot, base:base + cfg.block * cfg.d] = np.roll(pay, b)
            hc.arena[slot, base + cfg.block * cfg.d:base + sec] = sc_codes.astype(np.uint8)
    _gather_check(be, hc)


def test_merge_kernel_matches_oracle(be):
    import torch
    rng = np.random.default_rng(5)
    parts, rows, d = 5, 37, 128
    m = rng.normal(size=(parts, rows)).astype(np.float32) * 3
    l = rng.uniform(0.5, 50, size=(parts, rows)).astype(np.float32)
    l[1, :5] = 0.0
    m[1, :5] = -np.inf
    l[:, 7] = 0.0
    o = rng.normal(size=(parts, rows, d)).astype(np.float32)
    ref = oracle.merge_partials(m, l, o)
    md, ld, od = (torch.from_numpy(x).cuda() for x in (m, l, o))
    out = torch.zeros((rows, d), dtype=torch.int16, device="cuda")
    rc = be.merge(md.data_ptr(), ld.data_ptr(), od.data_ptr(), parts, rows, d, out.data_ptr(),
                  _stream())
    assert rc == 0
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    kvcase.assert_close_bf16(got, ref, what="merge")
    assert not got[7].any()


def test_append_then_decode(be):
    """Quantize-on-write then decode of the same pages: the decode sees the
    MX values the append produced (the oracle decodes the host copy)."""
    import torch
    cfg = replace(wl.C2, batch=4)
    hc = kvcase.build_case(cfg, seq_lens=[100, 37, 260, 17])
    dc = kvcase.DeviceCase(hc)
    # append one more token to every sequence (decode-step append); no
    # length is a multiple of 16, so every new token lands in a mapped page
    lens = hc.seq_lens
    mb = hc.plan.max_blocks
    pos = lens.copy()
    seq = np.arange(len(lens), dtype=np.int32)
    k = wl.normal_bf16(11, wl.ST_PK, 0, (len(pos), cfg.hkv, cfg.d))
    v = wl.normal_bf16(11, wl.ST_PV, 0, (len(pos), cfg.hkv, cfg.d))
    oracle.kv_append(k, v, seq, pos, hc.host_table(), mb, cfg.hkv, cfg.d, cfg.block, 1)
    # keep every device buffer referenced until the launch has completed
    kd = torch.from_numpy(k.view(np.int16).copy()).cuda()
    vd = torch.from_numpy(v.view(np.int16).copy()).cuda()
    sd = torch.from_numpy(seq).cuda()
    pd = torch.from_numpy(pos).cuda()
    rc = be.append(k=kd.data_ptr(), v=vd.data_ptr(), token_seq=sd.data_ptr(),
                   token_pos=pd.data_ptr(), num_tokens=len(seq), num_seqs=len(lens),
                   block_tables=dc.table.data_ptr(), max_blocks_per_seq=mb,
                   num_kv_heads=cfg.hkv, head_dim=cfg.d, block_size=16, kv_dtype=1,
                   stream=_stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert np.array_equal(dc.arena.cpu().numpy(), hc.arena), "append differs from oracle"
    new_lens = hc.seq_lens.copy()
    new_lens[seq] += 1
    hc.seq_lens = new_lens
    dc.seq_lens.copy_(torch.from_numpy(new_lens))
    rc = be.decode_v2(**dc.decode_kwargs(stream=_stream()))
    assert rc == 0
    kvcase.assert_close_bf16(dc.out_host(), hc.oracle_decode(), what="append+decode")
