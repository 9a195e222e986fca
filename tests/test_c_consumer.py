# SPDX-License-Identifier: Apache-2.0
"""tests/c/abi_consumer.c: a plain C program (no Python in the loop) links
libkllm_gpu and drives it as the reference's reactor drives its backend:
v1 decode on 128-token BF16 pages, v2 on 16-token BF16 pages, and v2 on
MX-FP8 pages the append kernel wrote, each against a double-precision
attention over the same cache values."""
from __future__ import annotations

import os
import subprocess

import pytest

import kllm_b200 as kb

HERE = os.path.dirname(os.path.abspath(__file__))


def _build(tmp_path) -> str:
    kb.load()                                   # the library exists
    lib_dir = os.path.dirname(kb.LIB_PATH)
    exe = str(tmp_path / "abi_consumer")
    subprocess.run(["gcc", "-std=c11", "-O2", "-Wall", "-Wextra", "-Werror", "-I",
                    os.path.dirname(kb.HEADER_PATH), os.path.join(HERE, "c", "abi_consumer.c"),
                    "-L", lib_dir, "-lkllm_gpu", f"-Wl,-rpath,{lib_dir}", "-lm", "-o", exe],
                   check=True)
    return exe


def _gpu_present() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_gpu_present(), reason="checks the no-device exit")
def test_builds_and_reports_no_device(tmp_path):
    out = subprocess.run([_build(tmp_path)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 77 and "skipped" in out.stdout


@pytest.mark.gpu
def test_c_caller_decodes(tmp_path):
    env = dict(os.environ, KLLM_GPU_DEVICE=os.environ.get("KLLM_GPU_DEVICE", "0"))
    out = subprocess.run([_build(tmp_path)], capture_output=True, text=True, timeout=300,
                         env=env)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.count(" ok ") == 3, out.stdout
