# SPDX-License-Identifier: Apache-2.0
"""Host logic: seeded generator, context-length draws, page plans."""
from __future__ import annotations

import numpy as np

from kllm_b200 import workloads as wl


def test_generator_is_deterministic_and_normal():
    a = wl.normal_bf16(0, wl.ST_K, 0, (4096,))
    b = wl.normal_bf16(0, wl.ST_K, 0, (4096,))
    assert np.array_equal(a, b)
    # counter-based: any window regenerates identically
    assert np.array_equal(wl.normal_bf16(0, wl.ST_K, 1000, (96,)), a[1000:1096])
    z = wl.normals(wl.stream_key(0, wl.ST_K), 0, 200000)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01
    assert not np.array_equal(a, wl.normal_bf16(1, wl.ST_K, 0, (4096,)))


def test_bf16_rounding_is_rne():
    x = np.array([1.0, 1 + 2 ** -8, 1 + 3 * 2 ** -8, -2.5, 0.0, 3.0e38], np.float32)
    got = wl.f32_to_bf16(x)
    assert got.tolist() == [0x3F80, 0x3F80, 0x3F82, 0xC020, 0x0000, 0x7F62]


def test_context_lengths_match_configs():
    c1 = wl.context_lengths(wl.C1)
    assert c1.min() >= 64 and c1.max() <= 512 and len(c1) == 8
    c2 = wl.context_lengths(wl.C2)
    assert c2.min() >= 512 and c2.max() <= 4096
    c3 = wl.context_lengths(wl.C3)
    assert c3.min() >= 128 and c3.max() <= 16384 and len(c3) == 256
    # log-uniform: the median sits near the geometric mean sqrt(128*16384) = 1448
    assert 900 < np.median(c3) < 2300
    assert wl.context_lengths(wl.C4).tolist() == [131072]


def test_page_plan_is_a_permutation():
    lens = wl.context_lengths(wl.C1)
    plan = wl.plan_pages(wl.C1, lens)
    used = plan.slots[plan.slots >= 0]
    assert len(np.unique(used)) == len(used) == plan.pages_used
    assert used.max() < plan.n_slots == 512
    pages = (lens + 15) // 16
    for s, p in enumerate(pages):
        assert (plan.slots[s, :p] >= 0).all() and (plan.slots[s, p:] < 0).all()
    t = wl.block_table(plan, wl.C1, 1 << 20)
    assert t.dtype.itemsize == 24
    assert (t["k"][plan.slots >= 0] % 16 == 0).all()


def test_algorithmic_bytes_mx():
    # 2,304 B per token per layer at 8 kv heads, d 128 (MX-FP8)
    assert wl.C2.kv_bytes_per_token() == 2304
    lens = np.array([16, 32], np.int32)
    b = wl.algorithmic_bytes(wl.C2, lens)
    assert b == 48 * 2304 + 2 * 32 * 128 * 4 + 3 * 24 + 2 * 4
