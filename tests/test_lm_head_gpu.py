# SPDX-License-Identifier: Apache-2.0
"""GPU vocabulary projection and sampling (kllm_gpu_lm_head_sample) against
the oracle: logits within the fp32 summation-order bound, greedy tokens
exact (the first maximum, ties included), temperature and top-k tokens
equal to the oracle's draw on the same logits except where r lies within
rounding of a cumulative boundary."""
from __future__ import annotations

import numpy as np
import pytest

import tablecase  # noqa: F401  (paths)
import oracle
import kllm_b200 as kb
from kllm_b200 import workloads as wl

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    import torch
    b = kb.Backend()
    assert b.backend == kb.KLLM_GPU_CUDA
    torch.cuda.set_stream(b.torch_stream())
    yield b
    torch.cuda.synchronize()
    torch.cuda.set_stream(torch.cuda.default_stream())
    b.close()


def _case(R, H, V, seed, dup=False):
    rng = np.random.default_rng(seed)
    h = wl.f32_to_bf16(rng.standard_normal((R, H)).astype(np.float32))
    w = wl.f32_to_bf16((rng.standard_normal((V, H)) * (1.5 / np.sqrt(H))).astype(np.float32))
    if dup:   # exact ties: vocabulary rows repeated, one of them made dominant for row 0
        w[V // 2] = w[3]
        w[V - 1] = w[3]
        w[3] = wl.f32_to_bf16(wl.bf16_to_f32(h[0]) * np.float32(0.05))
        w[V // 2] = w[3]
        w[V - 2] = w[3]
    return h, w


def _run(be, h, w, method, temp, topk, uni, want_logits=True):
    import torch
    R, H = h.shape
    V = w.shape[0]
    dev = "cuda"
    dh = torch.from_numpy(h.view(np.int16).copy()).to(dev)
    dw = torch.from_numpy(w.view(np.int16).copy()).to(dev)
    logits = torch.full((R, V), float("nan"), dtype=torch.float32, device=dev)
    tok = torch.full((R,), -1, dtype=torch.int32, device=dev)
    ws_b = be.lib.kllm_gpu_lm_head_workspace_size(R, V)
    ws = torch.zeros(ws_b, dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    dm = torch.from_numpy(np.asarray(method, np.int32)).to(dev) if method is not None else None
    dt = torch.from_numpy(np.asarray(temp, np.float32)).to(dev)
    dk = torch.from_numpy(np.asarray(topk, np.int32)).to(dev)
    du = torch.from_numpy(np.asarray(uni, np.float32)).to(dev)
    rc = be.lm_head(hidden=dh.data_ptr(), weight=dw.data_ptr(), num_rows=R, hidden_dim=H,
                    vocab=V, logits=logits.data_ptr() if want_logits else None,
                    method=dm.data_ptr() if dm is not None else None,
                    temperature=dt.data_ptr(), top_k=dk.data_ptr(), uniform=du.data_ptr(),
                    tokens=tok.data_ptr(), workspace=ws.data_ptr(), workspace_bytes=ws_b,
                    err_word=err.data_ptr(), stream=torch.cuda.current_stream().cuda_stream)
    assert rc == 0, (rc, be.stats().last_cuda_error)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return logits.cpu().numpy(), tok.cpu().numpy()


def _check_logits(h, w, got, rng, n_ids=384):
    V = w.shape[0]
    ids = np.unique(np.concatenate([rng.integers(0, V, n_ids), [0, V - 1]])).astype(np.int32)
    want = oracle.lm_head_logits(h, w, ids)
    absum = np.abs(wl.bf16_to_f32(h)).astype(np.float64) @ \
        np.abs(wl.bf16_to_f32(w[ids])).astype(np.float64).T
    bound = 3e-5 * absum + 1e-6      # fp32 sums in a different order
    assert (np.abs(got[:, ids] - want) <= bound).all()


def _cum_ok(lg, tok, t, r):
    """tok is where the float64 running sum of exp((l - max) / t) crosses
    r x total, within 1e-5 of the total (rounding of the two orders)."""
    x = np.exp((lg.astype(np.float64) - lg.max()) / t)
    c = np.cumsum(x) / x.sum()
    lo = c[tok - 1] if tok > 0 else 0.0
    return lo <= r + 1e-5 and c[tok] >= r - 1e-5


@pytest.mark.parametrize("R,H,V", [(1, 64, 1000), (5, 256, 1003), (128, 512, 2048),
                                   (129, 512, 4099), (256, 1024, 8192), (4, 256, 128256),
                                   (3, 128, 21000)])
def test_logits_and_greedy(be, R, H, V):
    """On 148 SMs: small vocabularies run every tile as two halves; 128,256
    rows (501 tiles) split only the last wave's 57; 21,000 rows (83 tiles)
    split none."""
    h, w = _case(R, H, V, R * 7 + V)
    logits, tok = _run(be, h, w, None, np.zeros(R), np.zeros(R), np.zeros(R))
    _check_logits(h, w, logits, np.random.default_rng(V))
    for r in range(R):
        assert tok[r] == int(np.argmax(logits[r])), r     # first maximum, exactly


def test_greedy_ties_take_the_first_index(be):
    R, H, V = 3, 256, 3000
    h, w = _case(R, H, V, 11, dup=True)
    logits, tok = _run(be, h, w, None, np.zeros(R), np.zeros(R), np.zeros(R))
    assert logits[0, 3] == logits[0, V // 2] == logits[0, V - 2]   # exact ties
    assert tok[0] == 3
    for r in range(R):
        assert tok[r] == int(np.argmax(logits[r]))


@pytest.mark.parametrize("R,H,V", [(16, 512, 5000), (200, 1024, 20000), (12, 256, 128256)])
def test_temperature_and_top_k(be, R, H, V):
    rng = np.random.default_rng(V)
    h, w = _case(R, H, V, 5 + R, dup=True)
    method = rng.choice([0, 1, 2, 3], R).astype(np.int32)
    temp = rng.choice([0.0, 0.4, 1.0, 2.0], R).astype(np.float32)
    topk = rng.choice([0, 1, 2, 7, 64, 1000, 1024, V, V + 5], R).astype(np.int32)
    uni = rng.random(R).astype(np.float32)
    uni[:3] = [0.0, 1.0, 0.999999]
    logits, tok = _run(be, h, w, method, temp, topk, uni)
    mismatch = 0
    for r in range(R):
        lg = logits[r]
        want = oracle.sample_token(lg, int(method[r]), float(temp[r]), int(topk[r]),
                                   float(uni[r]))
        if tok[r] == want:
            continue
        mismatch += 1
        m, t, k = int(method[r]), float(temp[r]), int(topk[r])
        assert m != 0 and t > 0, (r, m, t, k, tok[r], want)      # greedy is exact
        if m == 1 and 0 < k < V:
            order = np.lexsort((np.arange(V), -lg))[:k]          # (value desc, index asc)
            assert tok[r] in order
            pos = int(np.where(order == tok[r])[0][0])
            assert _cum_ok(lg[order], pos, t, float(uni[r])), (r, k)
        else:
            assert _cum_ok(lg, int(tok[r]), t, float(uni[r])), (r, m, t)
    assert mismatch <= max(1, R // 20), mismatch


def test_top_k_ties_order(be):
    """Row 0's dominant logit appears at indices 3, V/2 and V-2: top-1 is
    index 3, and a top-3 draw with a tiny temperature can only pick among
    the three tied ones."""
    R, H, V = 2, 256, 3000
    h, w = _case(R, H, V, 21, dup=True)
    logits, tok = _run(be, h, w, [1, 1], [1.0, 1.0], [1, 3], [0.5, 0.5])
    assert tok[0] == 3
    logits, tok = _run(be, h, w, [1, 1], [1e-3, 1e-3], [3, 3], [0.7, 0.1])
    assert tok[0] in (3, V // 2, V - 2)
    want = oracle.sample_token(logits[0], 1, 1e-3, 3, 0.7)
    assert tok[0] == want


def test_top_k_above_limit_is_refused(be):
    import torch
    R, H, V = 2, 64, 5000
    h, w = _case(R, H, V, 2)
    dh = torch.from_numpy(h.view(np.int16).copy()).cuda()
    dw = torch.from_numpy(w.view(np.int16).copy()).cuda()
    logits = torch.empty((R, V), dtype=torch.float32, device="cuda")
    tok = torch.zeros(R, dtype=torch.int32, device="cuda")
    ws_b = be.lib.kllm_gpu_lm_head_workspace_size(R, V)
    ws = torch.zeros(ws_b, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    m = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    k = torch.tensor([2000, 0], dtype=torch.int32, device="cuda")
    t = torch.tensor([1.0, 0.0], dtype=torch.float32, device="cuda")
    rc = be.lm_head(hidden=dh.data_ptr(), weight=dw.data_ptr(), num_rows=R, hidden_dim=H,
                    vocab=V, logits=logits.data_ptr(), method=m.data_ptr(),
                    temperature=t.data_ptr(), top_k=k.data_ptr(), tokens=tok.data_ptr(),
                    workspace=ws.data_ptr(), workspace_bytes=ws_b, err_word=err.data_ptr(),
                    stream=torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(tok[0].item()) == -1 and int(err.item()) == 0x10
    assert int(tok[1].item()) == int(np.argmax(logits[1].cpu().numpy()))


def test_rejects_bad_arguments(be):
    import torch
    d = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    p = d.data_ptr()
    assert be.lm_head(hidden=p, weight=p, num_rows=300, hidden_dim=64, vocab=10, tokens=p,
                      workspace=p, workspace_bytes=1 << 16) == kb.ENOSYS
    assert be.lm_head(hidden=p, weight=p, num_rows=2, hidden_dim=100, vocab=10, tokens=p,
                      workspace=p, workspace_bytes=1 << 16) == kb.ENOSYS
    assert be.lm_head(hidden=p, weight=p, num_rows=2, hidden_dim=64, vocab=10, tokens=p,
                      workspace=p, workspace_bytes=4) == kb.ENOSPC
    assert be.lm_head(hidden=p, weight=p, num_rows=2, hidden_dim=64, vocab=10, tokens=p,
                      method=p, workspace=p, workspace_bytes=1 << 16) == kb.EINVAL  # no logits
