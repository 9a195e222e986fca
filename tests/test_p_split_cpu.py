# SPDX-License-Identifier: Apache-2.0
"""Why the decode and prefill kernels write the softmax weights P as a bf16
pair (hi + lo) before the PV product, in a numpy emulation of that product
(fp32 P, bf16 V, float64 accumulation, bf16 output on both sides).

Inputs follow the decode test cases: scores with a spread of 0.5-6 (log2
units), V ~ N(0, 1) x U(0.5, 4) rounded to bf16, 2-511 keys per row. With P
rounded once to bf16 (8 significant bits) the output leaves the parity bound
|got - ref| <= 1e-3 + 2e-2 |ref| on a sizeable share of rows; with hi + lo
(P to about 2^-17) it stays well inside, the remaining difference being the
final bf16 rounding of the output."""
from __future__ import annotations

import numpy as np

ATOL, RTOL = 1e-3, 2e-2


def bf16(x) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even), returned as fp32 values."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def _rows(seed: int, n_rows: int):
    rng = np.random.default_rng(seed)
    for _ in range(n_rows):
        n = int(rng.integers(2, 512))
        s = (rng.standard_normal(n) * rng.uniform(0.5, 6)).astype(np.float32)
        v = bf16((rng.standard_normal((n, 128)) * rng.uniform(0.5, 4)).astype(np.float32))
        p = np.exp2(s - s.max()).astype(np.float32)      # fp32 weights, max 1
        yield p, v


def _ratio(p_used: np.ndarray, p: np.ndarray, v: np.ndarray) -> float:
    """Worst |out - ref| / (ATOL + RTOL |ref|) over the row's 128 outputs."""
    l = p.astype(np.float64).sum()                       # l sums the fp32 weights
    ref = bf16(((p.astype(np.float64)[:, None] * v).sum(0) / l).astype(np.float32))
    got = bf16(((p_used.astype(np.float64)[:, None] * v).sum(0) / l).astype(np.float32))
    ref = ref.astype(np.float64)
    return float(np.max(np.abs(got - ref) / (ATOL + RTOL * np.abs(ref))))


def test_hi_lo_split_keeps_the_bound_single_bf16_does_not():
    single, split = [], []
    for p, v in _rows(1, 300):
        hi = bf16(p)
        lo = bf16(p - hi)
        single.append(_ratio(hi, p, v))
        split.append(_ratio(hi.astype(np.float64) + lo, p, v))
    single, split = np.array(single), np.array(split)
    assert (single > 1.0).sum() >= 30, "one bf16 rounding of P should break the bound"
    assert split.max() < 0.5, f"hi + lo left the bound's half: {split.max():.3f}"
