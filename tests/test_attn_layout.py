"""The decode attention's shared-memory layout invariants, checked on the host (no GPU).

`attn_layout_check.cu` compiles the real `kernels_attn.cu` and evaluates its layout
functions for head dims 16-256, 1-8 heads per CTA, cluster sizes 1-8 and max_seq 16-8192:
score slots for every key, the packed probability bytes inside each head's own slots, the
chunked in-place writes landing only on slots already read, the value partials fitting the
ring, and the C4 / C5 bench shapes fitting 4 CTAs per SM.
"""
from __future__ import annotations

import subprocess
from pathlib import Path

import pytest

from llaccel_b200 import build as B

HERE = Path(__file__).resolve().parent


def test_decode_attention_layout_invariants(tmp_path):
    try:
        nvcc = B.nvcc()
    except RuntimeError:
        pytest.skip("nvcc not available")
    exe = tmp_path / "attn_layout_check"
    r = subprocess.run([nvcc, "-std=c++17", "-O1", "--expt-relaxed-constexpr", *B.ARCH_FLAGS, "-I", str(B.INCLUDE),
                        "-I", str(B.CSRC), str(HERE / "attn_layout_check.cu"), "-o", str(exe), "-lcuda"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-3000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-2000:]
    assert " 0 failures" in run.stdout
