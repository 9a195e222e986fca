# SPDX-License-Identifier: Apache-2.0
"""The C-ABI library loads, exports every symbol include/kllm_gpu.h
declares, and its structs have the layout C callers see. No compute call
is made without a GPU."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

import kllm_b200 as kb


def header_functions() -> list[str]:
    text = open(kb.HEADER_PATH).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kllm_gpu_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = kb.load()
    declared = header_functions()
    assert len(declared) >= 20
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"
    assert sorted(kb.symbols()) == declared, "binding and header disagree"


def test_reference_v1_symbols_present():
    """userspace/gpu/gpu_attention.h:43-62,70-73."""
    v1 = ["kllm_gpu_create", "kllm_gpu_destroy", "kllm_gpu_get_backend",
          "kllm_gpu_paged_attention", "kllm_gpu_malloc", "kllm_gpu_free",
          "kllm_gpu_memcpy_h2d", "kllm_gpu_get_stream", "kllm_gpu_paged_attention_cuda"]
    declared = header_functions()
    for n in v1:
        assert n in declared


def test_no_cpu_fallback_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", kb.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    names = [ln.split()[-1] for ln in out.splitlines() if ln.strip()]
    assert not [n for n in names if n.startswith(("orc_", "ref_"))], "oracle linked in"
    assert not any("ace_attention" in n for n in names)


STRUCTS = {
    "kllm_gpu_attention_params": kb.AttnParams,
    "kllm_gpu_attention_params_v2": kb.AttnParamsV2,
    "kllm_gpu_kv_append_params": kb.KvAppendParams,
    "kllm_gpu_gather_params": kb.GatherParams,
    "kllm_gpu_prefill_params": kb.PrefillParams,
    "kllm_gpu_table_build_params": kb.TableBuildParams,
    "kllm_gpu_lm_head_params": kb.LmHeadParams,
    "kllm_gpu_stats": kb.Stats,
}


def test_struct_layouts_match_c(tmp_path):
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "kllm_gpu.h"',
             "int main(void) {"]
    for cname, cls in STRUCTS.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof(struct {cname}));')
        for f, _ in cls._fields_:
            lines.append(f'printf("{cname}.{f} %zu\\n", offsetof(struct {cname}, {f}));')
    lines.append('printf("entry %zu\\n", sizeof(struct kllm_block_table_entry));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.dirname(kb.HEADER_PATH),
                    str(src), "-o", str(exe)], check=True)
    got = dict(ln.split() for ln in subprocess.run([str(exe)], capture_output=True, text=True,
                                                   check=True).stdout.splitlines())
    for cname, cls in STRUCTS.items():
        assert int(got[cname]) == ctypes.sizeof(cls), cname
        for f, _ in cls._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(cls, f).offset, f"{cname}.{f}"
    assert int(got["entry"]) == 24   # userspace/gpu/paged_attention.cu:18-22


def test_header_compiles_as_c_and_cxx(tmp_path):
    src = tmp_path / "h.c"
    src.write_text('#include "kllm_gpu.h"\nint x;\n')
    inc = os.path.dirname(kb.HEADER_PATH)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-c", "-I", inc, str(src), "-o",
                    str(tmp_path / "a.o")], check=True)
    subprocess.run(["g++", "-x", "c++", "-Wall", "-Werror", "-c", "-I", inc, str(src), "-o",
                    str(tmp_path / "b.o")], check=True)


def _gpu_present() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_gpu_present(), reason="checks the no-device behaviour")
def test_no_device_context_fails_loudly():
    lib = kb.load()
    ctx = lib.kllm_gpu_create()
    assert ctx, "create must return a context even without a device"
    try:
        assert lib.kllm_gpu_get_backend(ctx) == kb.KLLM_GPU_NONE
        p = kb.AttnParamsV2()
        p.struct_size = ctypes.sizeof(p)
        assert lib.kllm_gpu_paged_attention_v2(ctx, ctypes.byref(p)) == kb.ENODEV
        assert lib.kllm_gpu_paged_attention(ctx, ctypes.byref(kb.AttnParams())) == kb.ENODEV
        p.flags = 0x2           # not a defined flag: refused before anything else
        assert lib.kllm_gpu_paged_attention_v2(ctx, ctypes.byref(p)) == kb.EINVAL
        assert lib.kllm_gpu_malloc(ctx, 1024) is None
        assert lib.kllm_gpu_memcpy_h2d(ctx, None, None, 16) == kb.ENODEV
        # the table builder and lm_head refuse too, before any launch
        tp = kb.TableBuildParams()
        tp.struct_size = ctypes.sizeof(tp)
        assert lib.kllm_gpu_build_block_tables(ctx, ctypes.byref(tp)) == kb.ENODEV
        lp = kb.LmHeadParams()
        lp.struct_size = ctypes.sizeof(lp)
        assert lib.kllm_gpu_lm_head_sample(ctx, ctypes.byref(lp)) == kb.ENODEV
        # arena bookkeeping is host-side; tracing needs a device
        assert lib.kllm_gpu_register_arena(ctx, 4096, 1 << 20) == 0
        lib.kllm_gpu_clear_arenas(ctx)
        assert lib.kllm_gpu_trace_read(ctx, None, 0, None) == 0
        assert lib.kllm_gpu_trace_enable(ctx, 8) == kb.ENODEV
        st = kb.Stats()
        assert lib.kllm_gpu_get_stats(ctx, ctypes.byref(st)) == 0
        assert st.errors >= 4 and st.last_error == kb.ENODEV
    finally:
        lib.kllm_gpu_destroy(ctx)
    # workspace sizes are host arithmetic: midstates of 32 B per 16 tokens
    # (+1) per sequence; 12 B per (row, 256-row vocabulary tile) + 32
    assert lib.kllm_gpu_table_workspace_size(4, 8, 16) == 4 * (8 * 16 // 16 + 1) * 32
    assert lib.kllm_gpu_table_workspace_size(3, 5, 24) == 3 * (5 * 24 // 16 + 1) * 32
    assert lib.kllm_gpu_table_workspace_size(-1, 8, 16) == 0
    # a (max, sum, argmax) partial per row and 256-row vocabulary tile, twice
    # (the second halves of tiles computed as two halves)
    assert lib.kllm_gpu_lm_head_workspace_size(256, 128256) == 256 * 501 * 24 + 32
    assert lib.kllm_gpu_lm_head_workspace_size(0, 128256) == 0
    # the stateless v1 launcher validates before touching a device
    assert lib.kllm_gpu_paged_attention_cuda(None, None, None, None, 1, 32, 8, 96, 4,
                                             ctypes.c_float(0.1), None) == kb.ENOSYS
    assert lib.kllm_gpu_paged_attention_cuda(None, None, None, None, 1, 32, 8, 128, 4,
                                             ctypes.c_float(0.1), None) in (kb.EINVAL, kb.ENODEV)
