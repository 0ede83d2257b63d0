"""CPU tests of bench.py's host-side bookkeeping: which kernel function a plan step is
charged to (the roofline's dominant kernel), the committed ncu traffic lookup, the decode
launch count of each config and the seeded prompts."""
from __future__ import annotations

import sys

import numpy as np

from conftest import REPO

sys.path.insert(0, str(REPO))
import bench  # noqa: E402


def _prof():
    # llx_profile_decode rows: label "<kind>:<activation>", device ms, algorithmic bytes
    return [
        {"label": "embed:x0", "ms": 0.002, "bytes": 1e3},
        {"label": "rmsnorm:l0.h", "ms": 0.004, "bytes": 2e5},
        {"label": "linear_group:l0.q", "ms": 0.008, "bytes": 1.2e6},
        {"label": "rope_group:l0.qr", "ms": 0.0, "bytes": 0.0},  # folded into the attention
        {"label": "attention:l0.a", "ms": 0.017, "bytes": 2.1e7},
        {"label": "linear:l0.x1", "ms": 0.008, "bytes": 1.0e6},
        {"label": "gated:l0.f", "ms": 0.015, "bytes": 9.0e6},
        {"label": "linear_partial:l0.d", "ms": 0.011, "bytes": 5.0e6},
        {"label": "allreduce:l0.d", "ms": 0.037, "bytes": 4.0e6},
        {"label": "requant:l0.x2", "ms": 0.011, "bytes": 6.0e6},
        {"label": "argmax:logits", "ms": 0.003, "bytes": 1e3},
    ]


def test_by_kernel_charges_steps_to_their_kernel_functions():
    k = bench._by_kernel(_prof(), rows=128)
    assert k["k_linear_tc"]["n"] == 4  # q/k/v group, o, gate/up, the row-split partial
    assert abs(k["k_linear_tc"]["ms"] - (0.008 + 0.008 + 0.015 + 0.011)) < 1e-12
    assert k["k_attention_decode"] == {"n": 1, "ms": 0.017, "bytes": 2.1e7}
    assert k["ncclAllReduce"]["n"] == 1 and k["k_requant"]["n"] == 1
    assert "k_rope_group" not in k  # a folded step launches nothing and is not charged
    assert k["k_amax_finish"]["n"] == 1 and k["k_embed"]["n"] == 1


def test_by_kernel_small_batch_runs_linears_on_the_gemv():
    k = bench._by_kernel(_prof(), rows=1)
    assert "k_linear_tc" not in k
    assert k["k_gemv"]["n"] == 4
    k = bench._by_kernel(_prof(), rows=16)
    assert "k_gemv" not in k and k["k_linear_tc"]["n"] == 4


def test_by_kind_splits_linears_by_output_role():
    k = bench._by_kind(_prof())
    assert k["linear.x1"]["n"] == 1
    assert "rope_group" not in k
    assert list(k)[0] == "allreduce"  # sorted by time, largest first


def test_committed_traffic_lookup():
    e = bench._committed_traffic("c3", 128, "k_linear_tc")
    assert e is not None and e["bytes_per_launch"] > 1e6 and "profiles/" in e["source"]
    assert bench._committed_traffic("c3", 64, "k_linear_tc") is None
    assert bench._committed_traffic("c5", 256, "k_linear_tc") is None


def test_workload_decode_launches_per_config():
    class A:
        batch = prompt = decode = None
    for name, want_b, want_dec in [("c1", 1, 63), ("c2", 32, 127), ("c3", 128, 255), ("c4", 64, 127),
                                   ("c5", 256, 255)]:
        a = A()
        a.config = name
        cfg, w, n_dec = bench.workload(a)
        assert w["batch"] == want_b
        # the golden's launch rule: the last decode position has no successor to predict
        assert n_dec == want_dec == min(w["decode"], cfg.max_seq - w["prompt"] - 1)
    a = A()
    a.config, a.batch = "c5", 1
    assert bench.workload(a)[1]["batch"] == 1


def test_prompts_are_seeded_per_rank_and_in_vocab():
    p0 = bench.prompts_for(0, 4, 16, 50)
    assert p0.dtype == np.int32 and p0.shape == (4, 16)
    assert np.array_equal(p0, bench.prompts_for(0, 4, 16, 50))
    assert not np.array_equal(p0, bench.prompts_for(1, 4, 16, 50))
    assert p0.min() >= 0 and p0.max() < 50
