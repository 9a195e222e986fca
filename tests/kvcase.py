# SPDX-License-Identifier: Apache-2.0
"""Builds paged KV caches on the host (and on the GPU) for parity tests.

The host arena is laid out exactly as the device one; the block table for
the oracle holds host addresses, the one for the GPU holds device
addresses. MX pages are produced by the oracle's quantizer (the C
restatement pinned against the reference's codec).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace

import numpy as np

import oracle
from kllm_b200 import workloads as wl

ATOL, RTOL = 1e-3, 2e-2   # attention-output tolerance of the parity contract


def assert_close_bf16(got, ref, atol=ATOL, rtol=RTOL, what=""):
    g = wl.bf16_to_f32(np.asarray(got, dtype=np.uint16))
    r = wl.bf16_to_f32(np.asarray(ref, dtype=np.uint16))
    assert g.shape == r.shape, (g.shape, r.shape)
    assert np.all(np.isfinite(g)), f"{what}: non-finite output"
    err = np.abs(g - r)
    bad = err > atol + rtol * np.abs(r)
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.size} outside {atol}+{rtol}|ref|; first at "
            f"{tuple(i)}: got {g[tuple(i)]} ref {r[tuple(i)]}; max err {err.max():.3e}")


def assert_close_f32(got, ref, atol=ATOL, rtol=RTOL, what=""):
    g = np.asarray(got, dtype=np.float32)
    r = np.asarray(ref, dtype=np.float32)
    both_inf = np.isinf(g) & np.isinf(r) & (np.sign(g) == np.sign(r))
    err = np.where(both_inf, 0.0, np.abs(g - r))
    bad = ~(err <= atol + rtol * np.abs(np.where(both_inf, 0.0, r)))
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(f"{what}: {int(bad.sum())} bad; first {tuple(i)}: "
                             f"got {g[tuple(i)]} ref {r[tuple(i)]}")


@dataclass
class HostCase:
    cfg: wl.DecodeConfig
    seq_lens: np.ndarray
    plan: wl.PagePlan
    arena: np.ndarray          # uint8 [n_slots, slot_bytes]
    q: np.ndarray              # bf16 [layers?][B, Hq, D] for layer 0 .. layers-1
    valid: np.ndarray          # bool [B, max_blocks]

    def host_table(self) -> np.ndarray:
        return wl.block_table(self.plan, self.cfg, self.arena.ctypes.data, self.valid)

    def layer_off(self, layer: int) -> int:
        return layer * self.cfg.layer_stride()

    def oracle_decode(self, layer: int = 0, q=None):
        c = self.cfg
        return oracle.paged_decode(self.q[layer] if q is None else q, self.host_table(),
                                   self.seq_lens, c.hq, c.hkv, c.d, self.plan.max_blocks,
                                   c.scale, c.block, c.kv_dtype, self.layer_off(layer))

    def oracle_partials(self, layer: int = 0):
        c = self.cfg
        return oracle.paged_decode_partials(self.q[layer], self.host_table(), self.seq_lens,
                                            c.hq, c.hkv, c.d, self.plan.max_blocks, c.scale,
                                            c.block, c.kv_dtype, self.layer_off(layer))


def _pages_from_rows(cfg, rows_pay, rows_sc, n_pages, tail_fill):
    """[ntok, hkv, d(+scales)] token rows -> [n_pages, page_bytes] head sections."""
    bs, hkv = cfg.block, cfg.hkv
    ntok = rows_pay.shape[0]
    pad = n_pages * bs
    if cfg.kv_dtype == wl.KV_MX_FP8:
        pay = np.full((pad, hkv, cfg.d), tail_fill, dtype=np.uint8)
        sc = np.full((pad, hkv, cfg.d // 8), tail_fill, dtype=np.uint8)
        pay[:ntok] = rows_pay
        sc[:ntok] = rows_sc
        pay = pay.reshape(n_pages, bs, hkv, cfg.d).transpose(0, 2, 1, 3).reshape(
            n_pages, hkv, bs * cfg.d)
        sc = sc.reshape(n_pages, bs, hkv, cfg.d // 8).transpose(0, 2, 1, 3).reshape(
            n_pages, hkv, bs * cfg.d // 8)
        sec = np.concatenate([pay, sc], axis=2)
    else:
        kk = np.full((pad, hkv, cfg.d), tail_fill | (tail_fill << 8), dtype=np.uint16)
        kk[:ntok] = rows_pay
        sec = kk.reshape(n_pages, bs, hkv, cfg.d).transpose(0, 2, 1, 3).reshape(
            n_pages, hkv, bs * cfg.d).view(np.uint8)
    return np.ascontiguousarray(sec.reshape(n_pages, -1))


def build_case(cfg: wl.DecodeConfig, seed: int = 0, seq_lens=None, batch=None,
               invalid=None, tail_fill: int = 0xFF, max_blocks=None, layers=None,
               seq_ids=None) -> HostCase:
    """Seeded host case. ``invalid``: list of (seq, block) entries to mark invalid.
    ``tail_fill``: byte written past each sequence's last token (0xFF -> bf16 NaN,
    so masking of the partial last page is exercised). ``seq_ids``: global
    request ids whose K/V streams the sequences use (default 0..batch-1), so a
    shard of a batch holds the same data as the whole batch."""
    if batch is not None:
        cfg = replace(cfg, batch=batch)
    if layers is not None:
        cfg = replace(cfg, layers=layers)
    if seq_lens is None:
        seq_lens = wl.context_lengths(cfg, seed)
    seq_lens = np.asarray(seq_lens, dtype=np.int32)
    cfg = replace(cfg, batch=len(seq_lens))
    plan = wl.plan_pages(cfg, seq_lens, seed, max_blocks=max_blocks,
                         n_slots=None if cfg.arena_slots is None else
                         max(cfg.arena_slots, int(((np.maximum(seq_lens, 0) + cfg.block - 1)
                                                   // cfg.block).sum())))
    arena = np.zeros((plan.n_slots, cfg.slot_bytes()), dtype=np.uint8)
    ids = list(range(len(seq_lens))) if seq_ids is None else [int(x) for x in seq_ids]
    mult = wl.magnitudes(replace(cfg, batch=max(ids) + 1), seed)
    for layer in range(cfg.layers):
        loff = layer * cfg.layer_stride()
        for s, L in enumerate(seq_lens):
            if L <= 0:
                continue
            n_pages = (int(L) + cfg.block - 1) // cfg.block
            k, v = wl.seq_kv_bf16(cfg, ids[s], int(L), seed, layer, mult)
            for which, x in ((0, k), (1, v)):
                if cfg.kv_dtype == wl.KV_MX_FP8:
                    pay, sc = oracle.mx_quantize(x)
                else:
                    pay, sc = x, None
                pages = _pages_from_rows(cfg, pay, sc, n_pages, tail_fill)
                off = loff + which * cfg.page_bytes()
                arena[plan.slots[s, :n_pages], off:off + cfg.page_bytes()] = pages
    q = np.stack([wl.query_bf16(cfg, seed, layer) for layer in range(cfg.layers)])
    valid = plan.slots >= 0
    if invalid:
        for s, b in invalid:
            valid[s, b] = False
    return HostCase(cfg=cfg, seq_lens=seq_lens, plan=plan, arena=arena, q=q, valid=valid)


class DeviceCase:
    """The host case uploaded with torch (device memory only; every compute
    call goes through the C ABI)."""

    def __init__(self, hc: HostCase, device="cuda"):
        import torch
        self.hc = hc
        self.torch = torch
        self.arena = torch.from_numpy(hc.arena).to(device)
        base = self.arena.data_ptr()
        table = wl.block_table(hc.plan, hc.cfg, base, hc.valid)
        self.table = torch.from_numpy(table.view(np.uint8).copy()).to(device)
        self.seq_lens = torch.from_numpy(hc.seq_lens.copy()).to(device)
        self.q = torch.from_numpy(hc.q.view(np.int16).copy()).to(device)
        c = hc.cfg
        self.out = torch.zeros((c.batch, c.hq, c.d), dtype=torch.int16, device=device)

    def decode_kwargs(self, layer=0, **over):
        c = self.hc.cfg
        kw = dict(output=self.out.data_ptr(), query=self.q[layer].data_ptr(),
                  block_tables=self.table.data_ptr(), seq_lens=self.seq_lens.data_ptr(),
                  num_seqs=c.batch, num_heads=c.hq, num_kv_heads=c.hkv, head_dim=c.d,
                  max_blocks_per_seq=self.hc.plan.max_blocks, block_size=c.block,
                  kv_dtype=c.kv_dtype, layer=layer, layer_stride=c.layer_stride(),
                  scale=c.scale, split=1)
        kw.update(over)
        return kw

    def out_host(self) -> np.ndarray:
        self.torch.cuda.synchronize()
        return self.out.cpu().numpy().view(np.uint16)
