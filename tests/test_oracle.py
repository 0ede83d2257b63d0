"""Pins the CPU oracle (oracle/golden_oracle.py) to the reference: committed golden
vectors made by the reference's own code, and the reference tests' known answers
(tests/python/test_golden_primitives.py, test_rounding_boundaries.py, test_golden_e2e.py)."""
from __future__ import annotations

import json
import math

import numpy as np
import pytest

from conftest import GOLDEN, QGRAPH_FIXTURES
from oracle import golden_oracle as O


def test_luts_match_reference_tables():
    ref = json.loads((GOLDEN / "luts.json").read_text())
    assert O.SIG.tolist() == ref["SIG"]
    assert O.EXPI.tolist() == ref["EXPI"]
    assert O.EXPF.tolist() == ref["EXPF"]
    assert O.SIG[128] == 32768 and O.SIG[256] == 65514


def test_primitive_vectors():
    p = np.load(GOLDEN / "primitives.npz")
    np.testing.assert_array_equal(O.rshr(p["rshr_v"], p["rshr_s"]), p["rshr_out"])
    np.testing.assert_array_equal(O.requant16(p["rq_acc"], p["rq_M"], p["rq_S"]), p["rq16_out"])
    np.testing.assert_array_equal(O.requant8(p["rq_acc"], p["rq_M"], p["rq_S"]), p["rq8_out"])
    xs = np.arange(-32768, 32768)
    for prm, want in zip(p["silu_params"], p["silu_out"]):
        np.testing.assert_array_equal(O.silu16(xs, *prm), want)
    a, b, sh = p["ew_a"], p["ew_b"], p["ew_sh"]
    np.testing.assert_array_equal(O.vmul(a, b, sh), p["vmul_out"])
    np.testing.assert_array_equal(O.vadd(a, b, sh), p["vadd_out"])
    np.testing.assert_array_equal(O.vquant(a, p["rq_M"], p["rq_S"]), p["vquant_out"])
    assert [O.isqrt48(int(t)) for t in p["isqrt_in"]] == p["isqrt_out"].tolist()
    for K in (32, 128, 576):
        eps_t, C, sh_post = p[f"rms{K}_params"]
        np.testing.assert_array_equal(O.rmsnorm(p[f"rms{K}_x"], p[f"rms{K}_g"], eps_t, C, sh_post), p[f"rms{K}_out"])
    for H, D in ((4, 32), (2, 64), (2, 128)):
        k = f"rope{H}x{D}"
        np.testing.assert_array_equal(O.rope(p[k + "_x"], H, D, p[k + "_cos"], p[k + "_sin"], 37), p[k + "_out"])
    for i in p["att_cases"]:
        Ms, Ss, Mo, So, pb = (int(v) for v in p[f"att{i}_params"])
        out = O.attention_head(p[f"att{i}_q"], p[f"att{i}_k"], p[f"att{i}_v"], Ms, Ss, Mo, So, pb)
        np.testing.assert_array_equal(out, p[f"att{i}_out"])


# ---- known answers restated from the reference's tests ----------------------------------
def test_rshr_known_answers():
    assert O.rshr(np.array([5, -5, -6, 7, 6, -7]), np.array([1, 1, 1, 2, 2, 0])).tolist() == [3, -2, -3, 2, 2, -7]
    vals = np.array([-(1 << 63), (1 << 63) - 1, -1, 0, 1], dtype=np.int64)
    for s in range(64):
        want = [int(v) if s == 0 else (int(v) + (1 << (s - 1))) >> s for v in vals]
        assert O.rshr(vals, s).tolist() == want


def test_udiv_and_saturation_known_answers():
    assert O.udiv(10, 3) == 3 and O.udiv(10, 0) == 10 and O.udiv(2**31, 65534) == 32769
    assert O.udiv(2**40, 1) == 0
    v = np.array([-10**9, -32769, -128, 0, 127, 128, 32767, 32768])
    assert O.sat8(v).tolist() == [-128, -128, -128, 0, 127, 127, 127, 127]
    assert O.sat16(v).tolist() == [-32768, -32768, -128, 0, 127, 128, 32767, 32767]


def test_elementwise_known_answers():
    a, b = np.array([1000, -1000, 32767]), np.array([1000, 1000, 32767])
    assert O.vmul(a, b, 10).tolist() == [977, -977, 32767]
    assert O.vadd(a, b, 1).tolist() == [1500, -500, 32767]
    assert O.vquant(np.array([32767, -32768, 100]), 2**30, 38).tolist() == [127, -128, 0]


def test_attention_known_answers():
    # the max-score key gets p = 65534
    assert int(O._probs(np.array([0]))[0]) == 65534
    # 171 equal keys with V = 127: legacy Q0.8 gives 85, wide Q0.15 gives 127
    assert int(O.attention_head(np.zeros(16), np.zeros((171, 16)), np.full((171, 16), 127), 1, 0, 1 << 30, 38)[0]) == 85
    assert int(O.attention_head(np.zeros(16), np.zeros((171, 16)), np.full((171, 16), 127), 1, 0, 1 << 30, 38, 15)[0]) == 127
    # constant values survive every length within one LSB (wide mode)
    for T in (1, 2, 3, 100, 255, 256):
        for val in (-128, -1, 0, 1, 127):
            out = O.attention_head(np.zeros(16), np.zeros((T, 16)), np.full((T, 16), val), 1, 0, 1 << 30, 38, 15)
            assert np.abs(out - val).max() <= 1
    # score offset invariance with the largest unsigned multiplier
    for pb in (8, 15):
        for D in (16, 64, 128):
            q = np.full(D, 127)
            keys = np.array([[-128] * D, [127] * D])
            vals = np.zeros((2, D))
            vals[:, 0] = [-127, 127]
            assert O.attention_head(q, keys, vals, 2**32 - 1, 0, 1 << 30, 38, pb)[0] == 127


def test_rmsnorm_zero_row_and_clamp():
    K = 32
    g = np.full(K, 16384)
    C = int(round(2.0**24 * math.sqrt(K)))
    assert np.all(O.rmsnorm(np.zeros((1, K), np.int64), g, 3, C, 20) == 0)
    y = O.rmsnorm(np.ones((1, K), np.int64), g, 0, C, 20)[0]
    assert np.all(y == O.sat16(O.rshr(np.array([16384 * 65535]), 20))[0])


# ---- whole-model golden records --------------------------------------------------------------
def _prompt_and_n(d):
    rec = json.loads((d / "golden.json").read_text())
    return rec, rec["prompt_tokens"], len(rec["generated"])


@pytest.mark.parametrize("name", QGRAPH_FIXTURES)
def test_oracle_generate_matches_reference_record(name):
    d = GOLDEN / name
    rec, prompt, n = _prompt_and_n(d)
    assert O.OracleModel(d).generate(prompt, n) == rec


@pytest.mark.parametrize("name", QGRAPH_FIXTURES)
def test_oracle_activations_match_reference(name):
    d = GOLDEN / name
    rec, prompt, n = _prompt_and_n(d)
    want = np.load(d / "acts.npz")
    acts: list = []
    O.OracleModel(d).generate(prompt, n, acts)
    assert want.files
    for key in want.files:
        i, kind, pos, act = key.split("|", 3)
        step = acts[int(i)]
        assert step["kind"] == kind and step["pos"] == int(pos)
        np.testing.assert_array_equal(step["acts"][act].astype(np.int32), want[key], err_msg=key)


def test_chunked_prefill_equals_sequential_decode():
    d = GOLDEN / "fx_v1"
    toks = np.random.default_rng(3).integers(0, 16, 21).tolist()
    a = O.OracleModel(d).prefill(toks)
    g = O.OracleModel(d)
    b = [g.decode(t, i) for i, t in enumerate(toks)]
    for x, y in zip(a, b):
        np.testing.assert_array_equal(x, y)


def test_fused_equals_unfused():
    for v1, v2 in (("fx_v1", "fx_v2"), ("c1_v1", "c1_v2")):
        prompt = list(range(10))
        assert O.OracleModel(GOLDEN / v1).generate(prompt, 16) == O.OracleModel(GOLDEN / v2).generate(prompt, 16)


def test_errors_mirror_reference():
    g = O.OracleModel(GOLDEN / "fx_v1")
    with pytest.raises(ValueError, match="max_seq"):
        g.generate(list(range(10)), 64)
    with pytest.raises(ValueError, match="empty prompt"):
        g.generate([], 3)
