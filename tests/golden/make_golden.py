# SPDX-License-Identifier: Apache-2.0
"""Generates tests/golden/golden.npz from the REFERENCE's own code.

Run in a checkout where the reference sources exist (oracle/Makefile builds
oracle/_ref from them):

    make -C oracle && python tests/golden/make_golden.py

Every output below is computed by the reference's compiled C
(userspace/compute/ace_attention.c, userspace/compute/mx_dequant.h) on
seeded synthetic inputs; the tests check the oracle restatement and the
GPU path against these bytes. Inputs are regenerated from their seeds at
test time; their SHA-256 is stored so a drift of the generator is caught.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "xpu-kllm_b200"), os.path.join(ROOT, "oracle"),
                os.path.join(ROOT, "tests")]

import oracle  # noqa: E402
import kvcase  # noqa: E402
from kllm_b200 import workloads as wl  # noqa: E402


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def gathered_hash(hc) -> str:
    """Hash of the logical K/V the block table exposes (address-independent)."""
    c = hc.cfg
    t = hc.host_table()
    parts = []
    for s in range(c.batch):
        for h in range(c.hkv):
            k, v = oracle.gather(t[s], hc.plan.max_blocks, int(hc.seq_lens[s]), h, c.hkv, c.d,
                                 c.block, c.kv_dtype)
            parts += [k, v]
    return sha(*parts)


def ref_decode(hc):
    r = oracle.ref()
    c = hc.cfg
    out, *_ = oracle.harness_decode(r, "ref", hc.q[0], hc.host_table(), hc.seq_lens, c.hq,
                                    c.hkv, c.d, hc.plan.max_blocks, c.scale, c.block,
                                    c.kv_dtype, 0, 1)
    return out


def main():
    r = oracle.ref()
    if r is None:
        raise SystemExit("oracle/_ref not built: the reference sources are needed")
    meta = {"generator": "tests/golden/make_golden.py", "isa_level": int(r.ref_ace_probe()),
            "ref_lib": os.path.basename(oracle.ref_path())}
    g = {}

    # C1: BF16 paged decode, batch 8, 32q/8kv, d 128, 16-token pages, 512 slots
    hc1 = kvcase.build_case(wl.C1)
    g["c1_out"] = ref_decode(hc1)
    meta["c1"] = {"seq_lens": hc1.seq_lens.tolist(), "q_sha": sha(hc1.q),
                  "kv_sha": gathered_hash(hc1)}

    # C2 shape, first 4 sequences: MX-FP8 pages decoded with the reference decoder
    hc2 = kvcase.build_case(wl.C2, batch=4)
    g["c2b4_out"] = ref_decode(hc2)
    meta["c2b4"] = {"seq_lens": hc2.seq_lens.tolist(), "q_sha": sha(hc2.q),
                    "kv_sha": gathered_hash(hc2)}

    # E4M3 decoder, all 256 codes (mx_dequant.h:30-55)
    g["e4m3_decode"] = np.array([r.ref_fp8_e4m3_to_f32(c) for c in range(256)], np.float32)

    # mx_quant_to_bf16 (mx_dequant.h:105-136) on seeded inputs with zero blocks
    x = wl.normals(wl.stream_key(0, 99), 0, 4096).astype(np.float32)
    x *= np.repeat(np.float32(2.0) ** np.arange(-20, 12, dtype=np.float32), 128)[:4096]
    x[:8] = 0.0
    x[8:16] = -0.0
    data = np.zeros(4096, np.uint16)
    scales = np.zeros(512, np.uint8)
    r.ref_mx_quant_to_bf16(oracle.ptr(x), oracle.ptr(data), oracle.ptr(scales), 4096)
    g["compat_in"] = x
    g["compat_data"] = data
    g["compat_scales"] = scales

    # Known answer from tests/test_e2e_latency.c:170-172,190,226-237: 4 kv heads,
    # dim 64, MHA, seq_len 4, scale 1/8, K = 1.0 (0x3F80), V = 0.5 (0x3F00), q = 1.0
    k = np.full((16, 4, 64), 0x3F80, np.uint16)
    v = np.full((16, 4, 64), 0x3F00, np.uint16)
    q = np.full((1, 4, 64), 0x3F80, np.uint16)
    g["kat_e2e_out"] = oracle.attention(q, k, v, 4, 64, 4, 1, 1.0 / 8.0, use_ref=True)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **g)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote", {k: v.shape for k, v in g.items()})


if __name__ == "__main__":
    main()
