# SPDX-License-Identifier: Apache-2.0
"""The oracle's vocabulary projection and samplers on the CPU. The samplers
restate userspace/decode/decode_loop.c:58-183 with the uniform draw passed
in; they are pinned token for token against the reference's own functions
compiled from that file (oracle/_ref/libkllm_ref_sampling.so), with the
reference's rand() seeded so both see the same draw."""
from __future__ import annotations

import numpy as np
import pytest

import tablecase  # noqa: F401  (puts oracle/ on the path)
import oracle
from kllm_b200 import workloads as wl

needs_ref = pytest.mark.skipif(oracle.ref_sampling_lib() is None,
                               reason="reference sampling library not built")


def _logits(rng, v, kind):
    if kind == "normal":
        return rng.standard_normal(v).astype(np.float32) * 3
    if kind == "ties":          # few distinct values: many exact ties, at the top too
        return np.round(rng.standard_normal(v) * 2).astype(np.float32)
    if kind == "peaked":
        x = rng.standard_normal(v).astype(np.float32)
        x[rng.integers(0, v)] += 30.0
        return x
    raise ValueError(kind)


@needs_ref
@pytest.mark.parametrize("kind", ["normal", "ties", "peaked"])
def test_samplers_match_reference(kind):
    rng = np.random.default_rng(hash(kind) & 0xFFFF)
    n = 0
    for v in (7, 1000, 5003):
        for method in (0, 1, 2, 3, 9):
            for t in (0.0, -1.0, 0.3, 1.0, 2.5):
                for k in (0, 1, 2, 5, 50, v - 1, v, v + 3):
                    lg = _logits(rng, v, kind)
                    seed = int(rng.integers(1, 2**31 - 1))
                    want, r = oracle.ref_sample_with_seed(lg, method, t, k, seed)
                    got = oracle.sample_token(lg, method, t, k, r)
                    assert got == want, (v, method, t, k, kind)
                    n += 1
    assert n > 500


def test_greedy_first_maximum():
    lg = np.array([1, 5, 2, 5, 5, -1], np.float32)
    assert oracle.sample_token(lg, 0, 0.0, 0, 0.5) == 1
    # temperature <= 0 and top-k with T <= 0 are greedy too (decode_loop.c:77-78)
    assert oracle.sample_token(lg, 3, 0.0, 0, 0.9) == 1
    assert oracle.sample_token(lg, 1, 0.0, 3, 0.9) == 1


def test_lm_head_logits_vs_float64():
    rng = np.random.default_rng(3)
    h = wl.f32_to_bf16(rng.standard_normal((3, 256)).astype(np.float32))
    w = wl.f32_to_bf16((rng.standard_normal((50, 256)) / 16).astype(np.float32))
    got = oracle.lm_head_logits(h, w)
    want = wl.bf16_to_f32(h).astype(np.float64) @ wl.bf16_to_f32(w).astype(np.float64).T
    assert np.allclose(got, want, rtol=1e-5, atol=1e-5)
    ids = np.array([49, 0, 7], np.int32)
    assert np.array_equal(oracle.lm_head_logits(h, w, ids), got[:, ids])
