# SPDX-License-Identifier: Apache-2.0
"""Pins the oracle (C restatement) to the reference: golden fixtures made by
the reference's own code, and - where oracle/_ref was built from the
reference sources - the reference functions themselves."""
from __future__ import annotations

import numpy as np
import pytest

import golden
import kvcase
import oracle
from kllm_b200 import workloads as wl

G = golden.load()
META = golden.meta()


def test_e4m3_decode_matches_reference_all_codes():
    ours = oracle.e4m3_decode_table()
    ref = G["e4m3_decode"]
    assert np.array_equal(ours.view(np.uint32), ref.view(np.uint32))
    assert ref[0x7F] == 480.0 and ref[0xFF] == -480.0   # no NaN in the reference decoder
    assert ref[0x01] == 2.0 ** -9 and ref[0x08] == 2.0 ** -6


def test_e4m3_encode_round_trips_every_finite_code():
    o = oracle.orc()
    for c in range(256):
        if c & 0x7F == 0x7F:
            continue                      # 480 saturates to 448 by design
        v = o.orc_e4m3_decode(c)
        e = o.orc_e4m3_encode(v)
        if c == 0x80:
            assert e == 0x80
        else:
            assert e == c, (hex(c), v, hex(e))


def test_e4m3_encode_rounding_is_nearest_even_and_saturating():
    o = oracle.orc()
    dec = oracle.e4m3_decode_table()
    pos = np.sort(dec[:0x7F])             # 0 .. 448
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(0, 460, 20000), rng.uniform(0, 0.02, 20000),
                         (pos[1:] + pos[:-1]) / 2])   # exact midpoints
    for x in xs.astype(np.float32):
        e = o.orc_e4m3_encode(float(x))
        v = dec[e]
        # nearest representable (<= 448)
        d = np.abs(pos - x)
        best = d.min()
        assert abs(v - x) == best, (x, v)
        if np.count_nonzero(d == best) == 2:   # tie -> even mantissa
            assert e & 1 == 0, (x, hex(e))
    assert o.orc_e4m3_encode(1e9) == 0x7E and o.orc_e4m3_encode(-1e9) == 0xFE
    assert o.orc_e4m3_encode(470.0) == 0x7E


def test_scale_code_is_smallest_code_at_least_amax_over_448():
    o = oracle.orc()
    dec = oracle.e4m3_decode_table()
    rng = np.random.default_rng(1)
    for amax in np.concatenate([rng.uniform(0, 1e3, 5000), 2.0 ** rng.uniform(-40, 17, 5000),
                                [0.0, 448.0 * 448.0, 1e9]]).astype(np.float32):
        c = o.orc_mx_scale_code(float(amax))
        if amax == 0:
            assert c == 0
            continue
        t = np.float32(amax) / np.float32(448.0)
        if t > 448:
            assert c == 0x7E
            continue
        assert dec[c] >= t
        assert c == 1 or dec[c - 1] < t


def test_compat_quantizer_bit_exact_vs_reference_golden():
    x = G["compat_in"]
    data = np.zeros(4096, np.uint16)
    sc = np.zeros(512, np.uint8)
    oracle.orc().orc_mx_quantize_bf16_compat(oracle.ptr(x), oracle.ptr(data), oracle.ptr(sc),
                                             4096)
    assert np.array_equal(data, G["compat_data"])
    assert np.array_equal(sc, G["compat_scales"])
    assert set(np.unique(sc)) <= {0, 64}   # the reference's stub scale byte


def test_kat_e2e_latency_fixture():
    """tests/test_e2e_latency.c:170-172: K=1.0, V=0.5 -> every output 0.5."""
    assert np.all(G["kat_e2e_out"] == 0x3F00)
    k = np.full((16, 4, 64), 0x3F80, np.uint16)
    v = np.full((16, 4, 64), 0x3F00, np.uint16)
    q = np.full((1, 4, 64), 0x3F80, np.uint16)
    out = oracle.attention(q, k, v, 4, 64, 4, 1, 1.0 / 8.0)
    assert np.array_equal(out, G["kat_e2e_out"])


def test_attention_rejects_like_reference():
    q = np.zeros((1, 1, 8), np.uint16)
    with pytest.raises(ValueError):
        oracle.attention(q, q, q, 1, 8, 0, 1, 1.0)   # seq_len == 0 -> -1 (ace_attention.c:241)


@pytest.mark.parametrize("name", ["c1", "c2b4"])
def test_paged_decode_matches_reference_golden(name):
    cfg = wl.C1 if name == "c1" else wl.C2
    hc = kvcase.build_case(cfg, batch=None if name == "c1" else 4)
    m = META[name]
    assert hc.seq_lens.tolist() == m["seq_lens"]
    from golden.make_golden import gathered_hash, sha
    assert sha(hc.q) == m["q_sha"], "query generator drifted"
    assert gathered_hash(hc) == m["kv_sha"], "KV generator / quantizer drifted"
    kvcase.assert_close_bf16(hc.oracle_decode(), G[f"{name}_out"], what=name)
    # the restatement and the reference agree almost everywhere to the bit
    assert (hc.oracle_decode() == G[f"{name}_out"]).mean() > 0.99


def test_merge_of_split_context_equals_whole():
    hc = kvcase.build_case(wl.C2, batch=3, seq_lens=[2000, 33, 700])
    c = hc.cfg
    t = hc.host_table()
    whole = hc.oracle_decode()
    cut = 40  # pages
    parts = []
    for lo, hi in ((0, cut), (cut, hc.plan.max_blocks)):
        tt = np.zeros_like(t)
        tt[:, : hi - lo] = t[:, lo:hi]
        lens = np.clip(hc.seq_lens - lo * c.block, 0, (hi - lo) * c.block).astype(np.int32)
        parts.append(oracle.paged_decode_partials(hc.q[0], tt, lens, c.hq, c.hkv, c.d,
                                                  hc.plan.max_blocks, c.scale, c.block,
                                                  c.kv_dtype))
    m = np.stack([p[0] for p in parts])
    l = np.stack([p[1] for p in parts])
    o = np.stack([p[2] for p in parts])
    merged = oracle.merge_partials(m, l, o).reshape(whole.shape)
    kvcase.assert_close_bf16(merged, whole, what="merged halves")


@pytest.mark.skipif(oracle.ref() is None, reason="reference sources absent (oracle/_ref)")
class TestAgainstReferenceBuild:
    def test_decoder_all_codes(self):
        r = oracle.ref()
        ref = np.array([r.ref_fp8_e4m3_to_f32(c) for c in range(256)], np.float32)
        assert np.array_equal(ref.view(np.uint32), oracle.e4m3_decode_table().view(np.uint32))

    def test_compat_quantizer_random(self):
        r = oracle.ref()
        rng = np.random.default_rng(7)
        for scale in (1e-30, 1e-3, 1.0, 1e3, 1e30):
            x = (rng.normal(size=8192) * scale).astype(np.float32)
            x[rng.integers(0, 8192, 300)] = 0.0
            a, b = np.zeros(8192, np.uint16), np.zeros(8192, np.uint16)
            sa, sb = np.zeros(1024, np.uint8), np.zeros(1024, np.uint8)
            r.ref_mx_quant_to_bf16(oracle.ptr(x), oracle.ptr(a), oracle.ptr(sa), 8192)
            oracle.orc().orc_mx_quantize_bf16_compat(oracle.ptr(x), oracle.ptr(b),
                                                     oracle.ptr(sb), 8192)
            assert np.array_equal(a, b) and np.array_equal(sa, sb)

    @pytest.mark.parametrize("g,d,n", [(1, 64, 1), (4, 128, 300), (8, 128, 1000), (4, 64, 17)])
    def test_attention_random(self, g, d, n):
        q = wl.normal_bf16(1, 1, 0, (g, 1, d))
        k = wl.normal_bf16(1, 2, 0, (n, 1, d), 3.0)
        v = wl.normal_bf16(1, 3, 0, (n, 1, d))
        a = oracle.attention(q, k, v, 1, d, n, g, d ** -0.5, use_ref=True)
        b = oracle.attention(q, k, v, 1, d, n, g, d ** -0.5)
        kvcase.assert_close_bf16(b, a, what="orc vs ref attention")

    def test_harness_reference_equals_port(self):
        hc = kvcase.build_case(wl.C2, batch=3)
        c = hc.cfg
        args = (hc.q[0], hc.host_table(), hc.seq_lens, c.hq, c.hkv, c.d, hc.plan.max_blocks,
                c.scale, c.block, c.kv_dtype, 0, 4)
        a = oracle.harness_decode(oracle.ref(), "ref", *args)[0]
        b = oracle.harness_decode(oracle.orc(), "orc", *args)[0]
        kvcase.assert_close_bf16(b, a, what="harness")
