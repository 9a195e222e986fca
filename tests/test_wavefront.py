# SPDX-License-Identifier: Apache-2.0
"""KV block arrival into VRAM behind the reference's wavefront interface
(userspace/gpu/nvme_ep_wavefront.h; the reference's submit/poll are stubs,
nvme_ep_wavefront.c:74-104). CPU: the library exports every symbol the
header declares, the structs have the reference's layout, and with no device
the context is refused instead of spinning. GPU: blocks resolved by key
through the store index land in device memory byte for byte; missing keys
and destinations outside this GPU's device memory (host memory, an unmapped
address) are reported as failed without being written; completions come back
in submit order; a full queue refuses instead of blocking; a wait with
nothing pending ends at its bound."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import kllm_b200 as kb
import tablecase as tc


def _gpu_present() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def test_exports_every_declared_symbol():
    lib = kb.load()
    text = re.sub(r"/\*.*?\*/", "", open(kb.WAVEFRONT_HEADER_PATH).read(), flags=re.S)
    declared = sorted(set(re.findall(r"\b(kllm_wavefront_\w+)\s*\(", text)))
    assert sorted(kb.wavefront_symbols()) == declared
    assert not [n for n in declared if not hasattr(lib, n)]


def test_struct_layouts(tmp_path):
    structs = {"kllm_wf_block_desc": kb.WfBlockDesc, "kllm_wavefront": kb.Wavefront,
               "kllm_wf_completion": kb.WfCompletion}
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "kllm_wavefront.h"',
             "int main(void) {"]
    for cname, cls in structs.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof(struct {cname}));')
        for f, _ in cls._fields_:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof(struct {cname}, {f}));')
    lines.append("return 0; }")
    src = tmp_path / "wf.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "wf"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I",
                    os.path.dirname(kb.HEADER_PATH), str(src), "-o", str(exe)], check=True)
    got = dict(ln.split() for ln in subprocess.run([str(exe)], capture_output=True, text=True,
                                                   check=True).stdout.splitlines())
    for cname, cls in structs.items():
        assert int(got[cname]) == ctypes.sizeof(cls), cname
        for f, _ in cls._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(cls, f).offset, f"{cname}.{f}"
    # the reference's sizes: 56-byte descriptors, 64 per wavefront
    assert int(got["kllm_wf_block_desc"]) == 56 and int(got["kllm_wavefront"]) == 3600


def test_bad_arguments_refused(tmp_path):
    lib = kb.load()
    assert lib.kllm_wavefront_create(str(tmp_path / "missing").encode()) is None
    store = tmp_path / "store"
    store.write_bytes(b"\0" * 4096)
    # out of range before any device is touched: block size 0 or above 1 GiB,
    # fewer than 2 or more than 64 staging buffers, a negative device
    for dev, mb, nbuf in ((0, 0, 8), (0, (1 << 30) + 1, 8), (0, 4096, 1), (0, 4096, 65),
                          (-1, 4096, 8)):
        assert lib.kllm_wavefront_create2(str(store).encode(), dev, mb, nbuf) is None
    assert lib.kllm_wavefront_submit(None, None) == -1
    assert lib.kllm_wavefront_poll(None, None, 0) == -1
    assert lib.kllm_wavefront_wait(None, None, 1, 0) == -1


@pytest.mark.skipif(_gpu_present(), reason="checks the no-device behaviour")
def test_no_device_refused(tmp_path):
    store = tmp_path / "store"
    store.write_bytes(b"\0" * 4096)
    assert kb.load().kllm_wavefront_create(str(store).encode()) is None


def _store(tmp_path, n_records, record_bytes, seed):
    rng = np.random.default_rng(seed)
    data = rng.integers(0, 256, (n_records, record_bytes), dtype=np.uint8)
    path = tmp_path / "kv_store.bin"
    path.write_bytes(b"\x5a" * 512 + data.tobytes())       # records start at offset 512
    keys = [rng.integers(0, 256, 32, dtype=np.uint8).tobytes() for _ in range(n_records + 50)]
    entries = tc.empty_index(1024)
    for r in range(n_records):
        tc.index_insert(entries, keys[r], r)
    return path, data, keys, entries


@pytest.mark.gpu
def test_blocks_arrive_in_vram(tmp_path):
    import torch
    lib = kb.load()
    R, RB = 300, 36864                                     # one 16-token MX K+V block pair
    path, data, keys, entries = _store(tmp_path, R, RB, 1)
    wf_ctx = lib.kllm_wavefront_create2(str(path).encode(), 0, 1 << 20, 4)
    assert wf_ctx
    try:
        assert lib.kllm_wavefront_set_index(wf_ctx, entries.ctypes.data, len(entries), RB,
                                            512) == 0
        dev = torch.zeros((R + 60) * RB, dtype=torch.uint8, device="cuda")
        base = dev.data_ptr()
        rng = np.random.default_rng(2)
        host_buf = np.zeros(RB, dtype=np.uint8)         # not a device destination
        want = {}                     # device slot -> record (or None: not checked)
        n_wf, expect = 9, []
        slot = 0
        for w in range(n_wf):
            wf = kb.Wavefront()
            nb = int(rng.integers(1, 65))
            wf.num_blocks, wf.flags, wf.sequence_id = nb, 2, 1000 + w
            failed = 0
            for i in range(nb):
                rec = int(rng.integers(0, R + 50))      # >= R: a key the store lacks
                d = wf.blocks[i]
                ctypes.memmove(d.obj_key, keys[rec], 32)
                d.vram_dest_addr = base + slot * RB
                d.block_size = RB if i % 7 else RB - 100  # a short block now and then
                bad_dst = w == 3 and i % 5 == 1
                if bad_dst:
                    d.vram_dest_addr = host_buf.ctypes.data if i % 2 else 4096
                want[slot] = (rec if rec < R and not bad_dst else None, d.block_size)
                failed += rec >= R or bad_dst
                slot = (slot + 1) % (R + 60)
            assert lib.kllm_wavefront_submit(wf_ctx, ctypes.byref(wf)) == 0
            expect.append((1000 + w, nb - failed, failed))
        got = []
        comp = (kb.WfCompletion * 16)()
        while len(got) < n_wf:
            n = lib.kllm_wavefront_wait(wf_ctx, comp, 16, 10000)
            assert n > 0, "no completion within 10 s"
            got += [(comp[i].sequence_id, comp[i].blocks_completed, comp[i].blocks_failed)
                    for i in range(n)]
        assert got == expect                            # submit order, exact counts
        assert lib.kllm_wavefront_error(wf_ctx) == 0
        assert not host_buf.any()
        torch.cuda.synchronize()
        host = dev.cpu().numpy().reshape(R + 60, RB)
        for s, (rec, nbytes) in want.items():
            if rec is None:
                continue
            assert np.array_equal(host[s, :nbytes], data[rec, :nbytes]), s
        # nothing pending: the wait ends at its bound with 0
        assert lib.kllm_wavefront_wait(wf_ctx, comp, 16, 50) == 0
        # 64 wavefronts in flight at most: the 65th is refused, not blocked on
        wf = kb.Wavefront()
        wf.num_blocks, wf.sequence_id = 1, 7
        ctypes.memmove(wf.blocks[0].obj_key, keys[0], 32)
        wf.blocks[0].vram_dest_addr, wf.blocks[0].block_size = base, RB
        rcs = [lib.kllm_wavefront_submit(wf_ctx, ctypes.byref(wf)) for _ in range(65)]
        assert rcs[:64] == [0] * 64 and rcs[64] == -1
        drained = 0
        while drained < 64:
            n = lib.kllm_wavefront_wait(wf_ctx, comp, 16, 10000)
            assert n > 0
            drained += n
    finally:
        lib.kllm_wavefront_destroy(wf_ctx)
