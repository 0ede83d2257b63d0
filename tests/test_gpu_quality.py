"""GPU: host-side dequantized logits of the CUDA backend agree with the reference's (north
star: within 1e-6 relative error; the integer logits are bit-exact, so the error is zero),
and the quality report over a CUDA record equals the reference verify tool's on C1."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
from llaccel_b200 import quality

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)


def test_dequantized_logits_and_quality_report():
    from llaccel_b200 import build
    build.build()
    from llaccel_b200.cuda_backend import CudaModel
    rec = json.loads((GOLDEN / "c1_v2" / "golden.json").read_text())
    q = np.load(GOLDEN / "c1_quality.npz")
    with CudaModel(GOLDEN / "c1_v2") as m:
        got = m.generate(rec["prompt_tokens"], len(rec["generated"]))
    E = rec["model"]["E_LOGIT"]
    ours = quality.dequantize_logits(got["logits_last_rows"], E)
    ref = np.array(rec["logits_last_rows"], dtype=np.float64) * 2.0 ** E
    rel = np.abs(ours - ref) / np.maximum(np.abs(ref), 2.0 ** E)
    assert rel.max() <= 1e-6
    r = quality.compare_record(got, q["fp32_logits"])
    np.testing.assert_allclose([x["cos"] for x in r["rows"]], q["cos"], rtol=0, atol=1e-12)
    assert [x["fp32_top1"] for x in r["rows"]] == q["top1_fp32"].tolist()
