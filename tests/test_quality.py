"""Quality report (llaccel_b200.quality) pinned to the reference's verify tool on config C1.

The fixture c1_quality.npz holds the reference's fp32 TinyLlama logits, teacher-forced on the
C1 golden token stream, and the reference's per-step cosine / top-1 values
(tests/golden/make_quality.py)."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
from llaccel_b200 import quality
from llaccel_b200.artefacts import ArchConfig

C1 = ArchConfig("c1", 128, 2, 4, 2, 32, 352, 512, 80, 1e4, 1e-5)


def _fixture():
    q = np.load(GOLDEN / "c1_quality.npz")
    rec = json.loads((GOLDEN / "c1_v2" / "golden.json").read_text())
    return q, rec


def test_dequantize_is_exact():
    rng = np.random.default_rng(0)
    v = rng.integers(-32768, 32768, 1000)
    for E in (-12, -6, 0, 3):
        d = quality.dequantize_logits(v, E)
        # exact: scaling back recovers the integers; float32 holds the value too
        np.testing.assert_array_equal(d / 2.0**E, v)
        np.testing.assert_array_equal(d.astype(np.float32).astype(np.float64), d)


def test_report_matches_reference_metrics():
    q, rec = _fixture()
    r = quality.compare_record(rec, q["fp32_logits"])
    np.testing.assert_allclose([x["cos"] for x in r["rows"]], q["cos"], rtol=0, atol=1e-12)
    assert [x["int_top1"] for x in r["rows"]] == q["top1_golden"].tolist()
    assert [x["fp32_top1"] for x in r["rows"]] == q["top1_fp32"].tolist()
    assert r["top1_agreement"] > 0.8 and r["mean_cosine"] > 0.99


def test_float_forward_matches_reference_fp32_model():
    torch = pytest.importorskip("torch")
    q, rec = _fixture()
    w = dict(np.load(GOLDEN / "c1_float.npz"))
    seq = rec["prompt_tokens"] + rec["generated"]
    got = quality.teacher_forced_logits(C1, w, seq)
    np.testing.assert_allclose(got, q["fp32_logits"], rtol=1e-4, atol=1e-5)
    # so the report from our float model agrees with the reference's too
    r = quality.compare_record(rec, got)
    assert [x["fp32_top1"] for x in r["rows"]] == q["top1_fp32"].tolist()
    np.testing.assert_allclose([x["cos"] for x in r["rows"]], q["cos"], rtol=0, atol=1e-6)
