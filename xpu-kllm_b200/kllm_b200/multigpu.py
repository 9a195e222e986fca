# SPDX-License-Identifier: Apache-2.0
"""Work partitioning across GPUs for the paged-attention path.

Two strategies, one process per GPU:

* request sharding (continuous batching): independent sequences are packed
  onto ranks by longest-processing-time first on their context length; no
  data moves between GPUs;
* split-KV for one long context: rank r owns a contiguous range of the
  sequence's pages, decodes it into (m, l, o) triples, and the triples of
  all ranks are merged with the log-sum-exp rule after one all-gather
  (``kllm_gpu_comm_merge`` over NCCL on GPUs; the same math on CPU ranks in
  the tests).

Neither strategy exists in the reference (it has no multi-GPU code); the
split follows the page granularity of its block table
(``userspace/gpu/paged_attention.cu:55-68``).
"""
from __future__ import annotations

import numpy as np


def lpt_shard(lens, n: int) -> list[list[int]]:
    """Requests -> ranks, longest first onto the least-loaded rank (ties:
    lowest rank). Returns each rank's request indices in ascending order."""
    lens = np.asarray(lens)
    if n <= 0:
        raise ValueError("need at least one rank")
    loads = np.zeros(n, dtype=np.int64)
    out: list[list[int]] = [[] for _ in range(n)]
    for s in np.argsort(-lens, kind="stable"):
        r = int(np.argmin(loads))
        out[r].append(int(s))
        loads[r] += max(int(lens[s]), 0)
    return [sorted(x) for x in out]


def imbalance(lens, shards) -> float:
    """max rank load / mean rank load (1.0 = perfect)."""
    lens = np.maximum(np.asarray(lens), 0)
    loads = np.array([lens[s].sum() for s in shards], dtype=np.float64)
    return float(loads.max() / loads.mean()) if loads.mean() > 0 else 1.0


def page_ranges(num_pages: int, n: int) -> list[tuple[int, int]]:
    """Contiguous page ranges [lo, hi) of one sequence for n ranks."""
    return [(num_pages * r // n, num_pages * (r + 1) // n) for r in range(n)]


def local_view(table_row: np.ndarray, seq_len: int, block_size: int, lo: int, hi: int):
    """The part of one sequence's block-table row a rank owns: its entries
    moved to the front (same row width) and the number of context tokens
    they hold."""
    t = np.zeros_like(table_row)
    t[: hi - lo] = table_row[lo:hi]
    local_len = int(np.clip(seq_len - lo * block_size, 0, (hi - lo) * block_size))
    return t, local_len


def merge_triples(m: np.ndarray, l: np.ndarray, o: np.ndarray) -> np.ndarray:
    """Log-sum-exp merge of stacked triples [parts][rows](, d) -> fp32 [rows, d]."""
    m = np.asarray(m, dtype=np.float64)
    l = np.asarray(l, dtype=np.float64)
    o = np.asarray(o, dtype=np.float64)
    live = l > 0
    mm = np.where(live, m, -np.inf).max(axis=0)
    w = np.where(live, l * np.exp(np.where(live, m, 0.0) - np.where(np.isfinite(mm), mm, 0.0)),
                 0.0)
    den = w.sum(axis=0)
    num = (w[..., None] * o).sum(axis=0)
    return np.where(den[:, None] > 0, num / np.where(den > 0, den, 1.0)[:, None], 0.0).astype(
        np.float32)
