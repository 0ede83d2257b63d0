"""Pins the artefact generator's quantizer (llaccel_b200/artefacts.py) to the reference's
refquant output: same float weights + calibration -> identical qgraph and weight blob."""
from __future__ import annotations

import json
import math

import numpy as np
import pytest

from conftest import GOLDEN
from llaccel_b200 import artefacts as A


def _c1_inputs():
    w = dict(np.load(GOLDEN / "c1_float.npz"))
    w = {k: v.astype(np.float64) for k, v in w.items()}
    calib = json.loads((GOLDEN / "c1_calib.json").read_text())
    cfg = {"dim": 128, "n_layers": 2, "n_heads": 4, "n_kv_heads": 2, "head_dim": 32, "ffn": 352, "vocab": 512,
           "max_seq": 80, "rope_base": 10000.0, "rms_eps": 1e-5}
    return cfg, w, calib


@pytest.mark.parametrize("fusion,ref", [(False, "c1_v1"), (True, "c1_v2")])
def test_quantizer_reproduces_refquant(fusion, ref):
    cfg, w, calib = _c1_inputs()
    g, blob = A.quantize(cfg, w, calib, None, fusion)
    want = json.loads((GOLDEN / ref / "qgraph.json").read_text())
    assert g["ops"] == want["ops"]
    assert g["tensors"] == want["tensors"]
    assert g["model"] == want["model"]
    assert g["exps"] == want["exps"] and g["scales"] == want["scales"]
    assert blob == (GOLDEN / ref / "qweights.bin").read_bytes()


def test_torch_weight_path_matches_numpy():
    torch = pytest.importorskip("torch")
    cfg, w, calib = _c1_inputs()
    wt = {k: torch.from_numpy(v.astype(np.float32)) for k, v in w.items()}
    g1, b1 = A.quantize(cfg, wt, calib, None, True)
    g2, b2 = A.quantize(cfg, w, calib, None, True)
    assert g1 == g2 and b1 == b2


def test_generator_is_deterministic_for_d128():
    """The committed d128_tiny qgraph (run through the reference golden by make_fixtures)
    re-quantizes identically from its seed and stored calibration."""
    d = GOLDEN / "d128_tiny"
    man = json.loads((d / "manifest.json").read_text())
    arch = A.ArchConfig(**man["arch"])
    W = A.init_weights(arch, man["seed"], "cpu")
    calib = json.loads((d / "calib.json").read_text())
    qcfg = {k: getattr(arch, k) for k in ("dim", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab",
                                          "max_seq", "rope_base", "rms_eps")}
    g, blob = A.quantize(qcfg, W, calib, None, man["fusion"])
    assert g == json.loads((d / "qgraph.json").read_text())
    assert blob == (d / "qweights.bin").read_bytes()


def test_normalize_mulshift_vectorised_equals_scalar():
    rng = np.random.default_rng(5)
    r = np.concatenate([10.0 ** rng.uniform(-20, 9, 2000), [1.0 - 2.0**-40, 2.0**-40, 2.0**-70, 0.5, 1.0]])
    got = A.normalize_mulshift_np(r)
    want = np.array([A.normalize_mulshift(float(x)) for x in r])
    np.testing.assert_array_equal(got, want)
    assert A.normalize_mulshift(1.0 - 2.0**-40) == (2**30, 30)
    assert A.normalize_mulshift(2.0**-70) == (0, 63)


def test_llround_half_away_from_zero():
    assert [A.llround(x) for x in (2.5, -2.5, 0.5, -0.5, 1.4999, 0.0)] == [3, -3, 1, -1, 1, 0]
    assert A.llround_np(np.array([2.5, -2.5, 0.49999999999999994])).tolist() == [3, -3, 0]
    assert A.i16_exponent(32767.0) == 0 and A.i16_exponent(1.0) == -14 and A.i16_exponent(0.0) == -15


def test_configs_are_valid_geometry():
    for name, c in A.CONFIGS.items():
        assert c.n_heads % c.n_kv_heads == 0
        assert c.dim % 16 == 0 and c.ffn % 16 == 0 and (c.n_kv_heads * c.head_dim) % 16 == 0
        w = A.WORKLOADS[name]
        assert w["prompt"] + w["decode"] <= c.max_seq
        assert c.max_seq % 16 == 0
